"""Failure detection of the data-parallel job, on the host (gloo, world size 2).

The reference has no in-process fault handling (its recovery is relaunching
whole jobs, examples/run_with_resume.sh:33-53); a data-parallel step built on
this package must at least turn a lost or stalled rank into an error on the
others instead of a hang. Every process group here (and in bench.py) is given
a short timeout, so a rank that stalls before a collective or that leaves the
job makes the surviving rank's next collective raise within a bounded time.
The failures are made on the host: a rank that sleeps, or that exits.
"""

from __future__ import annotations

import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2
TIMEOUT_S = 3.0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _put_and_exit(out, item) -> None:
    out.put(item)
    out.close()
    out.join_thread()  # flush the queue's feeder thread before the hard exit
    os._exit(0)  # leaves without destroying the group


def _worker(rank, port, mode, out):
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=TIMEOUT_S))
    grads = torch.ones(1024)
    dist.all_reduce(grads)  # one healthy step first
    if rank == 1:
        if mode == "stall":
            time.sleep(4 * TIMEOUT_S)  # misses the next collective
        _put_and_exit(out, (rank, "left", 0.0))
    t0 = time.monotonic()
    try:
        dist.all_reduce(grads)
        result = (rank, "no error", time.monotonic() - t0)
    except Exception as exc:  # noqa: BLE001 - the error is the result
        result = (rank, type(exc).__name__, time.monotonic() - t0)
    _put_and_exit(out, result)


@pytest.mark.parametrize("mode", ["stall", "exit"])
def test_lost_rank_turns_into_an_error_on_the_survivor(mode):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, mode, out)) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        results = dict((r, (what, dt)) for r, what, dt in (out.get(timeout=60) for _ in range(WORLD)))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    what, dt = results[0]
    assert what != "no error", "the survivor's collective completed without its peer"
    # bounded: the group timeout (stall) or the peer's closed connection (exit)
    assert dt <= 4 * TIMEOUT_S, f"{mode}: error after {dt:.1f} s"
