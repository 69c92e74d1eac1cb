"""GPU parity of the fused gate ops (``spikegpt_b200.fused.gate``,
``relu_square`` and ``residual_add``) against the eager PyTorch ops they
replace: ``torch.sigmoid(r) * x`` and ``torch.relu(k).square()`` on bf16, and
the float32 + bf16 residual add, with their autograd backward. Both compute the same float32 products with the same bf16
roundings, so outputs and gradients are compared bit for bit, including
special values (NaN, infinities, signed zeros), sizes that are not a
multiple of the 8-element vector, and an empty tensor."""

from __future__ import annotations

import pytest
import torch

from spikegpt_b200 import _capi
from spikegpt_b200.fused import gate, relu_square, residual_add

pytestmark = pytest.mark.gpu

SPECIAL = [float("nan"), float("inf"), float("-inf"), 0.0, -0.0, 88.0, -88.0, 1e-30, -3.0e38]


def _bf16(shape, seed, cuda, scale=3.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    t = (torch.randn(shape, generator=g) * scale).to(torch.bfloat16)
    flat = t.view(-1)
    for i, v in enumerate(SPECIAL[: flat.numel()]):
        flat[(7 * i) % flat.numel()] = v
    return t.to(cuda)


def _same(a, b):
    """Bitwise equality of bf16 tensors (NaNs of either sign compare equal)."""
    nan = torch.isnan(a)
    assert torch.equal(nan, torch.isnan(b))
    assert torch.equal(a[~nan].view(torch.int16), b[~nan].view(torch.int16))


@pytest.mark.parametrize("shape", [(4, 64, 128), (3, 37, 11), (1,), (0, 5), (2, 1023, 512)])
def test_gate_matches_eager(cuda, shape):
    r0, x0, g = _bf16(shape, 1, cuda), _bf16(shape, 2, cuda), _bf16(shape, 3, cuda, 1.0)
    r, x = r0.clone().requires_grad_(), x0.clone().requires_grad_()
    out = gate(r, x)
    out.backward(g)
    re, xe = r0.clone().requires_grad_(), x0.clone().requires_grad_()
    ref = torch.sigmoid(re) * xe
    ref.backward(g)
    _same(out.detach(), ref.detach())
    _same(r.grad, re.grad)
    _same(x.grad, xe.grad)


@pytest.mark.parametrize("shape", [(4, 64, 512), (5, 13), (7,), (0,), (2, 1023, 2048)])
def test_relu_square_matches_eager(cuda, shape):
    k0, g = _bf16(shape, 4, cuda), _bf16(shape, 5, cuda, 1.0)
    k = k0.clone().requires_grad_()
    out = relu_square(k)
    out.backward(g)
    ke = k0.clone().requires_grad_()
    ref = torch.relu(ke).square()
    ref.backward(g)
    _same(out.detach(), ref.detach())
    _same(k.grad, ke.grad)


def test_unaligned_views_and_errors(cuda):
    base = _bf16((1, 1001), 6, cuda)
    r, x = base[:, 1:], base[:, :-1]  # 2-byte offset views: copied to aligned storage
    _same(gate(r, x), torch.sigmoid(r) * x)
    _same(relu_square(r), torch.relu(r).square())
    with pytest.raises(ValueError):
        gate(r.float(), x)
    with pytest.raises(ValueError):
        relu_square(r.cpu())
    lib = _capi.lib()
    assert lib.gate_forward(None, None, None, 8, None) == _capi.WKV_ERR_INVALID_ARGUMENT
    assert lib.relu_square_forward(base.data_ptr() + 2, base.data_ptr(), 8, None) == _capi.WKV_ERR_INVALID_ARGUMENT
    assert lib.gate_backward(None, None, None, None, None, -1, None) == _capi.WKV_ERR_INVALID_ARGUMENT


def test_gate_kernels_are_counted(cuda):
    before = _capi.launch_counts()
    x = _bf16((8, 16), 7, cuda).requires_grad_()
    relu_square(gate(x, x)).sum().backward()
    after = _capi.launch_counts()
    for name in ("gate_fwd_kernel", "gate_bwd_kernel", "relu_square_fwd_kernel", "relu_square_bwd_kernel"):
        assert after[name] - before[name] == 1, name
    residual_add(torch.zeros(8, 16, device=cuda), x.detach())
    assert _capi.launch_counts()["residual_add_kernel"] - after["residual_add_kernel"] == 1


@pytest.mark.parametrize("shape", [(4, 64, 512), (3, 5, 7), (0, 3)])
def test_residual_add_matches_eager(cuda, shape):
    g = torch.Generator(device="cpu").manual_seed(8)
    x0 = (torch.randn(shape, generator=g) * 5).to(cuda)
    s0 = _bf16(shape, 9, cuda)
    go = torch.randn(shape, generator=g).to(cuda)
    x, s = x0.clone().requires_grad_(), s0.clone().requires_grad_()
    out = residual_add(x, s)
    out.backward(go)
    xe, se = x0.clone().requires_grad_(), s0.clone().requires_grad_()
    ref = xe + se
    ref.backward(go)
    assert ref.dtype == torch.float32
    nan = torch.isnan(ref)
    assert torch.equal(nan, torch.isnan(out))
    assert torch.equal(out.detach()[~nan].view(torch.int32), ref.detach()[~nan].view(torch.int32))
    assert torch.equal(x.grad, xe.grad)
    _same(s.grad, se.grad)
