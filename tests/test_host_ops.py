"""Host-side behaviour of the custom ops that needs no GPU: registration under
the reference's names and schemas, fake/meta shape propagation (what
torch.compile traces), shape validation messages, and failing loudly off-GPU."""

from __future__ import annotations

import pytest
import torch

import spikegpt_b200  # noqa: F401  (registers the ops)
from spikegpt_b200 import validate_wkv_inputs


def _meta(*shape, dtype=torch.float32):
    return torch.empty(*shape, device="meta", dtype=dtype)


@pytest.mark.parametrize("fwd,bwd", [("wkv_forward", "wkv_backward"), ("wkv_forward_bf16io", "wkv_backward_bf16io")])
def test_ops_registered_with_reference_schemas(fwd, bwd):
    f = getattr(torch.ops.myelin, fwd).default._schema
    b = getattr(torch.ops.myelin, bwd).default._schema
    assert str(f) == f"myelin::{fwd}(Tensor key, Tensor value, Tensor time_decay, Tensor time_first) -> Tensor"
    assert str(b) == f"myelin::{bwd}(Tensor grad_y, Tensor w, Tensor u, Tensor k, Tensor v) -> Tensor[]"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fake_impls_give_reference_output_shapes(dtype):
    y = torch.ops.myelin.wkv_forward_bf16io(_meta(2, 5, 8, dtype=dtype), _meta(2, 5, 8, dtype=dtype), _meta(8), _meta(8))
    assert y.shape == (2, 5, 8) and y.dtype == dtype
    gk, gv, gtd, gtf = torch.ops.myelin.wkv_backward(
        _meta(2, 5, 8, dtype=dtype), _meta(8), _meta(8), _meta(2, 5, 8, dtype=dtype), _meta(2, 5, 8, dtype=dtype)
    )
    assert gk.shape == gv.shape == (2, 5, 8) and gk.dtype == dtype
    assert gtd.shape == gtf.shape == (8,) and gtd.dtype == torch.float32


def test_cpu_tensors_fail_loudly():
    x = torch.zeros(2, 3, 4)
    with pytest.raises(NotImplementedError):
        torch.ops.myelin.wkv_forward(x, x, torch.zeros(4), torch.zeros(4))
    with pytest.raises(NotImplementedError):
        torch.ops.myelin.wkv_backward_bf16io(x, torch.zeros(4), torch.zeros(4), x, x)


def test_validation_messages_match_the_reference():
    k = torch.zeros(2, 4, 3)
    with pytest.raises(ValueError, match="same shape"):
        validate_wkv_inputs(k, torch.zeros(2, 4, 2), torch.zeros(3), torch.zeros(3))
    with pytest.raises(ValueError, match=r"shape \[B, T, C\]"):
        validate_wkv_inputs(torch.zeros(4, 3), torch.zeros(4, 3), torch.zeros(3), torch.zeros(3))
    with pytest.raises(ValueError, match="time_decay must have shape"):
        validate_wkv_inputs(k, k, torch.zeros(4), torch.zeros(3))
    with pytest.raises(ValueError, match="time_first must have shape"):
        validate_wkv_inputs(k, k, torch.zeros(3), torch.zeros(2))
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        validate_wkv_inputs(k, k, torch.zeros(3), torch.zeros(3))


def test_autograd_formula_traces_on_fake_tensors():
    """The registered backward (w = -exp(td), then the backward op) runs on meta
    tensors through the fake impls, as AOTAutograd traces it under torch.compile."""
    k = _meta(2, 6, 8).requires_grad_()
    v = _meta(2, 6, 8).requires_grad_()
    td = _meta(8).requires_grad_()
    tf = _meta(8).requires_grad_()
    y = torch.ops.myelin.wkv_forward(k, v, td, tf)
    y.sum().backward()
    assert k.grad.shape == k.shape and td.grad.shape == td.shape


def test_state_keeping_forward_traces_on_fake_tensors():
    """The wrappers' state-keeping forward and its backward (through the saved
    state) trace on meta tensors, as torch.compile's AOTAutograd does."""
    from spikegpt_b200 import weighted_key_value_triton_bf16io

    k = _meta(2, 37, 72, dtype=torch.bfloat16).requires_grad_()
    v = _meta(2, 37, 72, dtype=torch.bfloat16).requires_grad_()
    td = _meta(72).requires_grad_()
    tf = _meta(72).requires_grad_()
    y, state = torch.ops.spikegpt_b200.wkv_forward_with_state(k, v, td, tf)
    assert y.shape == k.shape and y.dtype == k.dtype and state.dtype == torch.uint8
    weighted_key_value_triton_bf16io(k, v, td, tf).sum().backward()
    assert k.grad.shape == k.shape and tf.grad.shape == tf.shape


@pytest.mark.parametrize("shape", [(64, 1024, 512), (1, 1, 1), (3, 17, 70), (0, 5, 8), (2, 0, 8), (5, 3072, 96)])
def test_state_size_formula_matches_the_library(shape):
    from spikegpt_b200 import _capi
    from spikegpt_b200._ops import state_nbytes

    for code in (_capi.DTYPE_F32, _capi.DTYPE_BF16):
        assert state_nbytes(*shape) >= int(_capi.lib().wkv_state_size(code, *shape))
        if all(shape):
            assert state_nbytes(*shape) == int(_capi.lib().wkv_state_size(code, *shape))


def test_dropin_install_aliases_reference_module_names(monkeypatch):
    import sys

    from spikegpt_b200 import dropin, wkv, wkv_bf16

    monkeypatch.delitem(sys.modules, "spikegpt.wkv_triton", raising=False)
    monkeypatch.delitem(sys.modules, "spikegpt.wkv_bf16", raising=False)
    dropin.install()
    assert sys.modules["spikegpt.wkv_triton"] is wkv
    assert sys.modules["spikegpt.wkv_bf16"] is wkv_bf16
    assert wkv.weighted_key_value_triton is wkv.weighted_key_value_cuda
    assert wkv_bf16.weighted_key_value_triton_bf16io is wkv_bf16.weighted_key_value_cuda_bf16io


def test_residual_add_backward_takes_the_handed_bf16_gradient():
    """residual_add's backward (host logic, CPU tensors): the bf16 copy of its
    output gradient that an ln_shift_mix backward left under that gradient's
    identity is used as the spikes' gradient and consumed; any other gradient
    is cast. The skip gradient goes to the paired op only with a token."""
    from types import SimpleNamespace

    from spikegpt_b200 import fused

    g = torch.randn(2, 3, 4)
    made = (g * 0 + 1).to(torch.bfloat16)  # a stand-in that differs from the cast
    fused._BF16_GRADS[id(g)] = (g, made)
    gx, gs, _ = fused._resid_grad(SimpleNamespace(token=0), g)
    assert gx is g and gs is made and id(g) not in fused._BF16_GRADS
    other = torch.randn(2, 3, 4)
    gx, gs, _ = fused._resid_grad(SimpleNamespace(token=0), other)
    assert torch.equal(gs, other.to(torch.bfloat16))
    gx, gs, _ = fused._resid_grad(SimpleNamespace(token=7), other)
    assert gx is None and fused._RESIDUAL_GRADS.pop(7) is other
    fused._BF16_GRADS[id(g)] = (g, made)
    fused.drop_residual_grads()  # what TrainStep does after each backward
    assert not fused._BF16_GRADS and not fused._RESIDUAL_GRADS
