"""spikegpt_b200.train.TrainStep: the data-parallel train step.

CPU (gloo, world size 2, eager mode, a small stand-in model with the same
``model(ids, targets) -> loss`` interface): the gradients are gathered into
one flat buffer that one all-reduce averages over the ranks (the parameters'
gradients are then views of it), and after a step both ranks hold the
parameters that one process gets from the whole batch (the gradient of the
batch-mean loss is the mean of the shards').

GPU: the SpikeGPT model stepped by the captured CUDA graph follows the eager
step of the same model from the same initial state: the same losses and
parameters (rounding differences only: a library GEMM may pick another
algorithm for buffers at other addresses), with two batches alternating
through the static input buffers after capture; and the gradients the graph
leaves in the flat buffer match a plain autograd backward.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F
from torch import nn

from spikegpt_b200.train import TrainStep

WORLD = 2


class _TinyLM(nn.Module):
    def __init__(self, vocab: int = 11, width: int = 6) -> None:
        super().__init__()
        self.emb = nn.Embedding(vocab, width)
        self.mix = nn.Linear(width, width)
        self.head = nn.Linear(width, vocab, bias=False)

    def forward(self, ids, targets):
        h = torch.tanh(self.mix(self.emb(ids)))
        logits = self.head(h)
        return F.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.reshape(-1))


def _batch(rows: int = 4, t: int = 5):
    rng = np.random.default_rng(3)
    ids = torch.as_tensor(rng.integers(0, 11, (rows, t + 1)))
    return ids[:, :-1].contiguous(), ids[:, 1:].contiguous()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out, overlap=True, bucket_mb=25.0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        torch.manual_seed(0)
        model = _TinyLM()
        opt = torch.optim.SGD(model.parameters(), lr=0.5)
        x, y = _batch()
        rows = x.shape[0] // world
        step = TrainStep(model, opt, (rows, x.shape[1]), device="cpu", autocast_dtype=None, graph=False,
                         overlap=overlap, bucket_mb=bucket_mb)
        nbuckets = len(step.buckets)
        for _ in range(2):
            step(x[rank * rows:(rank + 1) * rows], y[rank * rows:(rank + 1) * rows])
        lo, hi = step.grads.data_ptr(), step.grads.data_ptr() + step.grads.numel() * 4
        views = all(lo <= p.grad.data_ptr() < hi for p in model.parameters())
        out.put((rank, views, nbuckets, [p.detach().clone().numpy() for p in model.parameters()]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("overlap,bucket_mb,nbuckets", [(True, 25.0, 1), (True, 1e-4, 3), (False, 25.0, 1)],
                         ids=["one-bucket", "small-buckets", "after-backward"])
def test_gradients_average_over_gloo_ranks(overlap, bucket_mb, nbuckets):
    """Bucketed all-reduces during the backward (one bucket, or buckets of 26
    elements: three all-reduces in flight over the four parameters) and the
    single all-reduce after it give the same parameters as one process on the
    whole batch."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, out, overlap, bucket_mb)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = sorted(out.get(timeout=120) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    torch.manual_seed(0)
    model = _TinyLM()
    opt = torch.optim.SGD(model.parameters(), lr=0.5)
    x, y = _batch()
    for _ in range(2):
        opt.zero_grad()
        model(x, y).backward()
        opt.step()
    for rank, views, got_buckets, params in results:
        assert views, rank
        assert got_buckets == nbuckets
        for got, ref in zip(params, model.parameters()):
            np.testing.assert_allclose(got, ref.detach().numpy(), rtol=1e-5, atol=1e-6)


def test_single_process_step_matches_plain_loop():
    torch.manual_seed(0)
    a, b = _TinyLM(), _TinyLM()
    b.load_state_dict(a.state_dict())
    opt_a = torch.optim.AdamW(a.parameters(), lr=1e-2, weight_decay=0.1)
    opt_b = torch.optim.AdamW(b.parameters(), lr=1e-2, weight_decay=0.1)
    x, y = _batch()
    step = TrainStep(a, opt_a, tuple(x.shape), device="cpu", autocast_dtype=None, graph=False)
    for _ in range(3):
        la = step(x, y)
        opt_b.zero_grad()
        lb = b(x, y)
        lb.backward()
        opt_b.step()
        assert torch.equal(la, lb.detach())
    for pa, pb in zip(a.parameters(), b.parameters()):
        assert torch.equal(pa, pb)


def test_rejects_other_batch_shapes_and_cpu_graphs():
    model = _TinyLM()
    opt = torch.optim.SGD(model.parameters(), lr=0.1)
    with pytest.raises(ValueError):
        TrainStep(model, opt, (2, 5), device="cpu", graph=True)
    step = TrainStep(model, opt, (2, 5), device="cpu", autocast_dtype=None, graph=False)
    x, y = _batch()
    with pytest.raises(ValueError):
        step(x, y)


def _spikegpt(cuda, seed=0):
    from spikegpt_b200.model import SpikeGPT, SpikeGPTConfig

    torch.manual_seed(seed)
    return SpikeGPT(SpikeGPTConfig(vocab_size=256, context_length=256, n_layer=2, n_embd=128)).to(cuda)


@pytest.mark.gpu
def test_graph_replay_follows_eager_step(cuda):
    eager, graphed = _spikegpt(cuda), _spikegpt(cuda)
    # plain SGD: an update linear in the gradient, so rounding-level gradient
    # differences stay rounding-level in the parameters
    opt_e = torch.optim.SGD(eager.parameters(), lr=0.05)
    opt_g = torch.optim.SGD(graphed.parameters(), lr=0.05)
    gen = torch.Generator(device="cpu").manual_seed(4)
    batches = [torch.randint(0, 256, (4, 257), generator=gen).to(cuda) for _ in range(2)]
    step_e = TrainStep(eager, opt_e, (4, 256), device=cuda, graph=False)
    step_g = TrainStep(graphed, opt_g, (4, 256), device=cuda, graph=True)
    for i in range(6):
        ids = batches[i % 2]
        le = step_e(ids[:, :-1], ids[:, 1:]).item()
        lg = step_g(ids[:, :-1], ids[:, 1:]).item()
        assert abs(le - lg) <= 1e-4 * max(1.0, abs(le)), (i, le, lg)
    for (name, pe), pg in zip(eager.named_parameters(), graphed.parameters()):
        scale = max(float(pe.abs().max()), 1e-6)
        assert float((pe - pg).abs().max()) <= 1e-4 * scale, name
    step_g.release()


@pytest.mark.gpu
def test_graph_gradients_match_autograd(cuda):
    ref, graphed = _spikegpt(cuda, 7), _spikegpt(cuda, 7)
    opt = torch.optim.SGD(graphed.parameters(), lr=0.0)
    ids = torch.randint(0, 256, (2, 257), generator=torch.Generator(device="cpu").manual_seed(1)).to(cuda)
    step = TrainStep(graphed, opt, (2, 256), device=cuda, graph=True)
    step(ids[:, :-1], ids[:, 1:])
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = ref(ids[:, :-1], ids[:, 1:])
    loss.backward()
    for (name, pr), pg in zip(ref.named_parameters(), graphed.parameters()):
        scale = max(float(pr.grad.abs().max()), 1e-12)
        assert float((pr.grad - pg.grad).abs().max()) <= 1e-3 * scale, name
    step.release()


@pytest.mark.gpu
def test_weight_cache_matches_autocast_casts(cuda):
    """The step's one-kernel bf16 weight copies and widened bf16 weight
    gradients give autocast's per-weight casts' gradients."""
    plain, cached = _spikegpt(cuda, 11), _spikegpt(cuda, 11)
    ids = torch.randint(0, 256, (2, 257), generator=torch.Generator(device="cpu").manual_seed(2)).to(cuda)
    steps = [TrainStep(m, torch.optim.SGD(m.parameters(), lr=0.0), (2, 256), device=cuda, graph=False,
                       weight_cache=wc) for m, wc in ((plain, False), (cached, True))]
    assert steps[0].cache is None and steps[1].cache is not None
    losses = [float(s(ids[:, :-1], ids[:, 1:])) for s in steps]
    assert abs(losses[0] - losses[1]) <= 1e-6 * max(1.0, abs(losses[0])), losses
    for (name, pp), pc in zip(plain.named_parameters(), cached.parameters()):
        scale = max(float(pp.grad.abs().max()), 1e-12)
        assert float((pp.grad - pc.grad).abs().max()) <= 1e-3 * scale, name
    # the matmul weights are views of the flat buffer, their gradients too
    groups, head = cached.matmul_weights()
    for p in [q for g in groups for q in g]:
        assert p.data_ptr() >= steps[1].w32.data_ptr()
        assert p.grad.data_ptr() >= steps[1].grads.data_ptr()


@pytest.mark.gpu
def test_stacked_gradients_match_unbound_slices(cuda, monkeypatch):
    """With cached weights, the time-mixing core (_TimeCore) and the channel
    mixing's paired projections (_CachedPair) write their input gradients
    stacked; the loss and every gradient equal, bit for bit, those of the
    separate ops on unbound slices whose gradients autograd stacks."""
    import spikegpt_b200.model as model_mod

    ids = torch.randint(0, 256, (2, 257), generator=torch.Generator(device="cpu").manual_seed(4)).to(cuda)
    results = []
    for stacked in (False, True):
        monkeypatch.setattr(model_mod, "_STACKED_GRADS", stacked)
        m = _spikegpt(cuda, 17)
        step = TrainStep(m, torch.optim.SGD(m.parameters(), lr=0.0), (2, 256), device=cuda, graph=False)
        assert step.cache is not None
        loss = float(step(ids[:, :-1], ids[:, 1:]))
        results.append((loss, [p.grad.clone() for p in m.parameters()]))
    assert results[0][0] == results[1][0]
    for (name, _), g0, g1 in zip(m.named_parameters(), results[0][1], results[1][1]):
        assert torch.equal(g0, g1), name


@pytest.mark.gpu
def test_micro_batches_match_one_batch(cuda):
    """Two micro-batches on their own streams (replayed from the graph) give
    the one-batch step's loss and, up to the bf16 rounding of each micro-batch's
    weight gradients, its gradients."""
    one, two = _spikegpt(cuda, 13), _spikegpt(cuda, 13)
    ids = torch.randint(0, 256, (4, 257), generator=torch.Generator(device="cpu").manual_seed(5)).to(cuda)
    s1 = TrainStep(one, torch.optim.SGD(one.parameters(), lr=0.0), (4, 256), device=cuda, graph=True)
    s2 = TrainStep(two, torch.optim.SGD(two.parameters(), lr=0.0), (4, 256), device=cuda, graph=True,
                   micro_batches=2)
    for _ in range(2):  # the second replay rewrites every gradient the first wrote
        l1, l2 = float(s1(ids[:, :-1], ids[:, 1:])), float(s2(ids[:, :-1], ids[:, 1:]))
    assert abs(l1 - l2) <= 1e-4 * max(1.0, abs(l1)), (l1, l2)
    for (name, p1), p2 in zip(one.named_parameters(), two.parameters()):
        scale = max(float(p1.grad.abs().max()), 1e-12)
        assert float((p1.grad - p2.grad).abs().max()) <= 1e-2 * scale, name
    s1.release()
    s2.release()
    with pytest.raises(ValueError):
        TrainStep(_spikegpt(cuda), torch.optim.SGD(one.parameters(), lr=0.0), (3, 256), device=cuda,
                  graph=False, micro_batches=2)
