"""Multi-rank logic of the batch-sharded WKV job, on CPU with gloo (world size 2).

The per-rank compute here is the CPU oracle standing in for the GPU op (the
GPU path itself is covered by test_wkv_cuda.py, including the same shard-sum
invariant on one device); what is tested is the host-side plumbing a
data-parallel job uses: how the batch is split, that summing the per-channel
gradients of the shards over ranks gives the full-batch gradients, and the
max-over-ranks timing reduction bench.py uses.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from _wkvtest import config_inputs, scaled_err

from oracle import oracle
from spikegpt_b200.sharding import max_over_ranks, reduce_channel_grads, shard_range

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, b, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        k, v, td, tf, gy = config_inputs(b, 96, 70, seed=5, kscale=2.0)
        lo, hi = shard_range(b, world, rank)
        _, _, _, gtd, gtf = oracle.forward_backward(k[lo:hi], v[lo:hi], td, tf, gy[lo:hi])
        gtd_t, gtf_t = torch.as_tensor(gtd, dtype=torch.float32), torch.as_tensor(gtf, dtype=torch.float32)
        reduce_channel_grads(gtd_t, gtf_t)
        slowest = max_over_ranks(10.0 * (rank + 1))
        out.put((rank, lo, hi, gtd_t.numpy(), gtf_t.numpy(), slowest))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("b", [4, 5, 1])
def test_shard_gradients_sum_to_full_batch_over_gloo(b):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, b, out)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [out.get(timeout=120) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    k, v, td, tf, gy = config_inputs(b, 96, 70, seed=5, kscale=2.0)
    _, _, _, gtd, gtf = oracle.forward_backward(k, v, td, tf, gy)
    covered = []
    for rank, lo, hi, r_gtd, r_gtf, slowest in results:
        covered += list(range(lo, hi))
        # float32 all-reduce of float64 shard sums: float32 rounding
        assert scaled_err(r_gtd, gtd) < 1e-6, rank
        assert scaled_err(r_gtf, gtf) < 1e-6, rank
        assert slowest == 10.0 * WORLD
    assert covered == list(range(b))


def test_shard_range_splits_contiguously():
    for batch in range(0, 11):
        for world in range(1, 5):
            parts = [shard_range(batch, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == batch
            for (a0, a1), (b0, _) in zip(parts, parts[1:]):
                assert a1 == b0
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_single_process_helpers_are_identity():
    g = torch.arange(5, dtype=torch.float32)
    reduce_channel_grads(g)
    assert torch.equal(g, torch.arange(5, dtype=torch.float32))
    assert max_over_ranks(3.5) == 3.5
    np.testing.assert_array_equal(g.numpy(), np.arange(5, dtype=np.float32))
