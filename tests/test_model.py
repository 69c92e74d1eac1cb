"""SpikeGPT model and train step (spikegpt_b200.model) against the reference's
own model (golden vectors from tests/golden/make_golden_model.py).

CPU: parameter count and FLOPs of SpikeGPT-41M, the initial values of the
non-matrix parameters (decays, bonuses, mixing profiles) against the
reference's. GPU: with the reference's parameters loaded, the loss, logits and
every gradient in float32 (the model runs on this package's WKV and LIF
kernels, the reference on its CPU paths; both use the same spike rule, so the
comparison is to float32 rounding of the whole network: loss to 1e-5, logits
to 1e-4 and each gradient to 1e-3 of its own scale); a bf16-autocast train step; the
data-parallel invariant (the gradient of the batch mean is the mean of the
shards' gradients)."""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch
from _wkvtest import scaled_err

from spikegpt_b200.model import (SPIKEGPT_41M, SPIKEGPT_216M, SpikeGPT, SpikeGPTConfig, flops_per_token,
                                 parameter_count)

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "model_golden.npz")


def _golden_config() -> SpikeGPTConfig:
    v, ctx, nl, ne = (int(x) for x in GOLDEN["config"])
    return SpikeGPTConfig(vocab_size=v, context_length=ctx, n_layer=nl, n_embd=ne)


def _golden_model(device) -> SpikeGPT:
    torch.manual_seed(0)
    model = SpikeGPT(_golden_config())
    state = {k[len("param/"):]: torch.as_tensor(GOLDEN[k]) for k in GOLDEN.files if k.startswith("param/")}
    model.load_state_dict(state, strict=True)
    return model.to(device)


def test_41m_parameters_and_flops():
    model = SpikeGPT(SPIKEGPT_41M)
    assert parameter_count(model) == 41_226_240
    assert flops_per_token(SPIKEGPT_41M) == pytest.approx(246.2e6, rel=1e-3)


def test_216m_class_parameters():
    # 18 x 13 x 768^2 matrix weights + 2 x 50257 x 768 embedding and head + the vectors
    assert parameter_count(SpikeGPT(SPIKEGPT_216M)) == 215_368_704
    assert flops_per_token(SPIKEGPT_216M) == pytest.approx(1059.7e6, rel=1e-4)


def test_initial_values_match_reference():
    model = SpikeGPT(_golden_config())
    params = dict(model.named_parameters())
    checked = 0
    for key in GOLDEN.files:
        if not key.startswith("param/"):
            continue
        name = key[len("param/"):]
        if name.endswith(".weight") and GOLDEN[key].ndim == 2:
            continue  # matrices were redrawn by the golden script
        np.testing.assert_allclose(params[name].detach().numpy(), GOLDEN[key], rtol=1e-6, atol=1e-7,
                                   err_msg=name)
        checked += 1
    assert checked > 20


def test_shapes_and_errors():
    model = SpikeGPT(_golden_config())
    with pytest.raises(ValueError):
        model(torch.zeros(4, dtype=torch.long))
    with pytest.raises(ValueError):
        model(torch.zeros(1, 1000, dtype=torch.long))
    with pytest.raises(ValueError):
        SpikeGPTConfig(n_embd=0).validate()


@pytest.mark.gpu
def test_float32_parity_with_reference_model(cuda):
    model = _golden_model(cuda)
    ids = torch.as_tensor(GOLDEN["ids"]).to(cuda)
    logits = model(ids[:, :-1])
    loss = model(ids[:, :-1], ids[:, 1:])
    loss.backward()
    assert abs(loss.item() - float(GOLDEN["loss"])) <= 1e-5 * max(1.0, abs(float(GOLDEN["loss"])))
    assert scaled_err(logits.detach().cpu().numpy(), GOLDEN["logits"]) <= 1e-4
    for name, p in model.named_parameters():
        ref = GOLDEN[f"grad/{name}"]
        scale = max(float(np.abs(ref).max()), 1e-30)
        assert float(np.abs(p.grad.cpu().numpy() - ref).max()) <= 1e-3 * scale, name


@pytest.mark.gpu
def test_bf16_train_step(cuda):
    cfg = SpikeGPTConfig(vocab_size=256, context_length=256, n_layer=2, n_embd=128)
    torch.manual_seed(1)
    model = SpikeGPT(cfg).to(cuda)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3, weight_decay=0.1, fused=True)
    ids = torch.randint(0, 256, (4, 257), device=cuda)
    losses = []
    for _ in range(8):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(ids[:, :-1], ids[:, 1:])
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(loss.item())
    assert all(math.isfinite(x) for x in losses)
    assert abs(losses[0] - math.log(256)) < 0.05  # tiny initial weights: uniform prediction
    assert losses[-1] < losses[0]


@pytest.mark.gpu
def test_data_parallel_gradient_is_mean_of_shards(cuda):
    model = _golden_model(cuda)
    rng = np.random.default_rng(9)
    ids = torch.as_tensor(rng.integers(0, model.config.vocab_size, (4, model.config.context_length + 1))).to(cuda)

    def grads(batch):
        model.zero_grad(set_to_none=True)
        model(batch[:, :-1], batch[:, 1:]).backward()
        return {n: p.grad.detach().clone() for n, p in model.named_parameters()}

    full = grads(ids)
    a, b = grads(ids[:2]), grads(ids[2:])
    for n in full:
        ref = full[n].cpu().numpy()
        mean = ((a[n] + b[n]) / 2).cpu().numpy()
        assert scaled_err(mean, ref) <= 1e-4, n


@pytest.mark.gpu
def test_padded_head_matches_plain_projection(cuda):
    """The output projection of an unaligned vocabulary runs on a weight padded
    to 64 rows: logits and the weight's gradient are those of the plain
    projection (float32: to rounding of the GEMM's own order)."""
    from spikegpt_b200.model import _head

    g = torch.Generator(device="cpu").manual_seed(5)
    h = torch.randn(4, 33, 96, generator=g).to(cuda)
    w = torch.randn(50257 // 64 + 5, 96, generator=g).to(cuda).requires_grad_()  # 790 rows: not a multiple of 64
    w2 = w.detach().clone().requires_grad_()
    full, v = _head(h, w)
    assert v == w.shape[0] and full.shape[-1] % 64 == 0
    out = full[..., :v]
    ref = h @ w2.T
    assert out.shape == ref.shape
    go = torch.randn(out.shape, generator=g).to(cuda)
    out.backward(go)
    ref.backward(go)
    assert scaled_err(out.detach().cpu().numpy(), ref.detach().cpu().numpy()) <= 1e-5
    assert scaled_err(w.grad.cpu().numpy(), w2.grad.cpu().numpy()) <= 1e-5


def test_embedding_table_normalization_matches_per_token():
    """The spike and the first block's LayerNorm act row by row, so with V <=
    B*T the model applies them to the embedding table's rows before the lookup
    (the model's forward needs CUDA; this checks the front it changes, on
    CPU): the values equal the per-token order's bit for bit, and the
    gradients of the table and the LayerNorm agree to float32 rounding. The
    whole model stays pinned to the reference's by the GPU parity test."""
    import torch.nn.functional as F

    from spikegpt_b200.model import _HardSpike

    model = _golden_model("cpu")
    emb, ln0, slope = model.embedding, model.blocks[0].ln0, model.config.surrogate_slope
    ids = torch.as_tensor(GOLDEN["ids"])[:, :-1]
    assert model.config.vocab_size <= ids.numel()  # the model takes the table order here
    up = torch.randn(*ids.shape, emb.weight.shape[1], generator=torch.Generator().manual_seed(3))

    def run(table_order):
        model.zero_grad(set_to_none=True)
        if table_order:
            x = F.embedding(ids, ln0(_HardSpike.apply(slope * emb.weight)))
        else:
            x = ln0(_HardSpike.apply(slope * emb(ids)))
        (x * up).sum().backward()
        return x.detach(), [p.grad.clone() for p in (emb.weight, ln0.weight, ln0.bias)]

    (xt, gt), (xp, gp) = run(True), run(False)
    assert torch.equal(xt, xp)
    for a_, b_ in zip(gt, gp):
        scale = max(float(b_.abs().max()), 1e-30)
        assert float((a_ - b_).abs().max()) <= 1e-5 * scale
