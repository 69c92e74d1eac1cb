"""GPU parity of the fused LayerNorm + token-shift mixing op against the
eager float32 computation it replaces (LayerNorm, shift-mix, bf16 rounding):
outputs within one bf16 rounding (2e-2 relative), input and parameter
gradients within 1e-4 of their scale (float32 sums in a different order)."""

from __future__ import annotations

import contextlib

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from spikegpt_b200 import _capi
from spikegpt_b200.fused import ln_shift_mix

pytestmark = pytest.mark.gpu


def _eager(x, w, b, mixes, eps):
    h = F.layer_norm(x, (x.shape[-1],), w, b, eps)
    prev = F.pad(h[:, :-1], (0, 0, 1, 0))
    return [(h * m + prev * (1.0 - m)).to(torch.bfloat16) for m in mixes]


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / max(float(b.abs().max()), 1e-30))


# the last two shapes take 64 and 32 steps per CTA (the others 8)
@pytest.mark.parametrize("shape,n", [((2, 70, 128), 3), ((3, 200, 512), 3), ((1, 65, 512), 2), ((2, 33, 768), 3),
                                     ((1, 1, 256), 1), ((80, 1024, 128), 2), ((40, 1000, 128), 3)])
def test_forward_backward_match_eager(cuda, shape, n):
    g = torch.Generator(device="cpu").manual_seed(sum(shape) + n)
    b_, t, c = shape
    x = (torch.randn(shape, generator=g) * 2 + 0.5).to(cuda).requires_grad_()
    w = (1 + 0.3 * torch.randn(c, generator=g)).to(cuda).requires_grad_()
    b = (0.2 * torch.randn(c, generator=g)).to(cuda).requires_grad_()
    mixes = [torch.rand(1, 1, c, generator=g).to(cuda).requires_grad_() for _ in range(n)]
    grads = [torch.randn(shape, generator=g).to(cuda).to(torch.bfloat16) for _ in range(n)]

    outs = ln_shift_mix(x, w, b, mixes)
    torch.autograd.backward(outs, grads)
    got = [o.detach().float() for o in outs]
    gx, gw, gb, gm = x.grad.clone(), w.grad.clone(), b.grad.clone(), [m.grad.clone() for m in mixes]
    for p in [x, w, b, *mixes]:
        p.grad = None
    ref = _eager(x, w, b, mixes, 1e-5)
    torch.autograd.backward(ref, grads)
    for o, r in zip(got, ref):
        assert _rel(o, r.float()) <= 2e-2
    assert _rel(gx, x.grad) <= 1e-4
    assert _rel(gw, w.grad) <= 1e-4
    assert _rel(gb, b.grad) <= 1e-4
    for a, m in zip(gm, mixes):
        assert _rel(a, m.grad) <= 1e-4


def test_deterministic_parameter_gradients(cuda):
    x = torch.randn(4, 300, 512, device=cuda, requires_grad=True)
    w = torch.ones(512, device=cuda, requires_grad=True)
    b = torch.zeros(512, device=cuda, requires_grad=True)
    m = torch.rand(512, device=cuda, requires_grad=True)
    gr = torch.randn(4, 300, 512, device=cuda).to(torch.bfloat16)
    res = []
    for _ in range(2):
        (o,) = ln_shift_mix(x, w, b, [m])
        o.backward(gr)
        res.append((w.grad.clone(), m.grad.clone()))
        w.grad = m.grad = x.grad = None
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])


def test_errors(cuda):
    x = torch.randn(2, 8, 100, device=cuda)
    with pytest.raises(ValueError):
        ln_shift_mix(x, torch.ones(100, device=cuda), torch.zeros(100, device=cuda), [torch.zeros(100, device=cuda)])
    x = torch.randn(2, 8, 128, device=cuda)
    with pytest.raises(ValueError):
        ln_shift_mix(x, torch.ones(128, device=cuda), torch.zeros(128, device=cuda), [])


def test_kernels_are_counted(cuda):
    before = _capi.launch_counts()
    x = torch.randn(1, 64, 128, device=cuda, requires_grad=True)
    (o,) = ln_shift_mix(x, torch.ones(128, device=cuda), torch.zeros(128, device=cuda), [torch.rand(128, device=cuda)])
    o.float().sum().backward()
    torch.cuda.synchronize()
    after = _capi.launch_counts()
    for k in ("ln_mix_fwd_kernel", "ln_mix_bwd_kernel", "ln_mix_reduce_kernel"):
        assert after[k] > before.get(k, 0)


def test_residual_gradient_summed_in_kernel(cuda):
    """A sublayer closed by residual_add with the ln_shift_mix's token: the
    skip connection's gradient reaches x through the LayerNorm-mix backward
    kernel instead of autograd's sum, with the same value bit for bit."""
    from spikegpt_b200 import fused

    g = torch.Generator(device="cpu").manual_seed(21)
    shape = (3, 90, 256)
    x0 = (torch.randn(shape, generator=g) * 2).to(cuda)
    w = (1 + 0.3 * torch.randn(256, generator=g)).to(cuda)
    b = (0.2 * torch.randn(256, generator=g)).to(cuda)
    m = [torch.rand(1, 1, 256, generator=g).to(cuda) for _ in range(2)]
    go = torch.randn(shape, generator=g).to(cuda)

    def run(paired):
        x = x0.clone().requires_grad_()
        with fused.residual_handoff() if paired else contextlib.nullcontext():
            tok = fused.new_residual_token(x)
            assert (tok != 0) == paired
            xk, xr = fused.ln_shift_mix(x, w, b, m, 1e-5, tok)
            out = fused.residual_add(x, fused.gate(xk, xr), tok)
            out.backward(go)
        return x.grad

    assert torch.equal(run(True), run(False))
    assert fused.pending_residual_grads() == 0  # every handed-over gradient was consumed


def test_bf16_grad_copy_is_the_cast(cuda):
    """Asked for it, the LayerNorm-mix backward also writes grad x rounded to
    bf16, bit for bit grad_x.to(bfloat16); inside residual_handoff() the
    residual_add whose output is x takes it as the spikes' gradient, which then
    equals the eager cast of that add's output gradient."""
    from spikegpt_b200 import fused

    g = torch.Generator(device="cpu").manual_seed(23)
    shape = (2, 130, 512)
    x = torch.randn(shape, generator=g).to(cuda)
    w = (1 + 0.3 * torch.randn(512, generator=g)).to(cuda)
    b = (0.2 * torch.randn(512, generator=g)).to(cuda)
    mix = torch.rand(3, 512, generator=g).to(cuda)
    stacked, mean, rstd = torch.ops.spikegpt_b200.ln_shift_mix(x, w, b, mix, 1e-5, 0)
    gouts = [torch.randn(shape, generator=g).to(cuda).to(torch.bfloat16) for _ in range(3)]
    gres = torch.randn(shape, generator=g).to(cuda)
    for res in (None, gres):
        gx, _, _, _, gx16 = torch.ops.spikegpt_b200.ln_shift_mix_backward(gouts, x, w, b, mix, mean, rstd, res, True)
        assert torch.equal(gx16, gx.to(torch.bfloat16))
        gx_plain, *_, empty = torch.ops.spikegpt_b200.ln_shift_mix_backward(gouts, x, w, b, mix, mean, rstd, res)
        assert torch.equal(gx_plain, gx) and empty.numel() == 0

    # through autograd: spikes -> residual_add -> ln_shift_mix
    x0 = torch.randn(shape, generator=g).to(cuda)
    s0 = (torch.rand(shape, generator=g) < 0.3).to(torch.bfloat16).to(cuda)
    m = [torch.rand(1, 1, 512, generator=g).to(cuda) for _ in range(2)]
    go = [torch.randn(shape, generator=g).to(cuda).to(torch.bfloat16) for _ in range(2)]

    def run(handoff):
        spikes = s0.clone().requires_grad_()
        with fused.residual_handoff() if handoff else contextlib.nullcontext():
            out = fused.residual_add(x0, spikes, 0)
            xk, xr = fused.ln_shift_mix(out, w, b, m, 1e-5, 0)
            torch.autograd.backward([xk, xr], go)
        fused.drop_residual_grads()
        return spikes.grad

    ga, gb = run(True), run(False)
    assert ga.dtype == torch.bfloat16 and torch.equal(ga, gb)


def test_residual_token_only_inside_the_handoff_context(cuda):
    """Outside residual_handoff(), for inputs without grad, and under
    torch.compile no token is handed out, so a partial backward
    (torch.autograd.grad on a subset) loses no skip gradient."""
    from spikegpt_b200 import fused

    x = torch.randn(2, 8, 128, device=cuda, requires_grad=True)
    assert fused.new_residual_token(x) == 0
    with fused.residual_handoff():
        assert fused.new_residual_token(x.detach()) == 0
        assert fused.new_residual_token(x) != 0
    assert fused.new_residual_token(x) == 0
    w = torch.ones(128, device=cuda)
    b = torch.zeros(128, device=cuda)
    m = [torch.full((1, 1, 128), 0.5, device=cuda)]
    xk, = fused.ln_shift_mix(x, w, b, m, 1e-5, fused.new_residual_token(x))
    out = fused.residual_add(x, xk.float().to(torch.bfloat16), 0)
    (gx,) = torch.autograd.grad(out.sum(), [x])
    assert torch.isfinite(gx).all() and fused.pending_residual_grads() == 0
