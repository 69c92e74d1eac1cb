"""Recurrent (single-token) WKV step for generation.

The reference computes one generation step of the WKV recurrence inline in
``SpikeTimeMix.step`` (src/spikegpt/language.py:977-1013): after the key and
value projections it updates the state ``(numerator, denominator,
log_scale)`` (natural-log scale, in the dtype ``initial_state`` gives it at
language.py:957-975: the model dtype, or float32 under autocast) and
multiplies the WKV output by the receptance gate. ``weighted_key_value_step`` is that WKV part (lines 993-1010)
as one sm_100a kernel launch, with the same inputs, state and results, so a
model's ``step`` can call it in place of the inline arithmetic:

    wkv, numerator, denominator, log_scale = weighted_key_value_step(
        key, value, self.time_decay, self.time_first,
        state.numerator, state.denominator, state.log_scale)
    return self.output(receptance * wkv), SpikeTimeMixState(
        previous=inputs, numerator=numerator, denominator=denominator, log_scale=log_scale)

``weighted_key_value_step_`` updates the state tensors in place instead (no
allocation per token, for decode loops and CUDA graphs). There is no autograd
formula: generation runs without gradients, like the reference's step.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _capi
from ._ops import _CODES


def _check(key: Tensor, value: Tensor, time_decay: Tensor, time_first: Tensor, state: tuple[Tensor, ...]) -> None:
    if key.ndim != 2:
        raise ValueError(f"key must have shape [B, C]; got {tuple(key.shape)}")
    for name, t in (("value", value), ("numerator", state[0]), ("denominator", state[1]), ("log_scale", state[2])):
        if t.shape != key.shape:
            raise ValueError(f"{name} must have the shape of key {tuple(key.shape)}; got {tuple(t.shape)}")
    if value.dtype != key.dtype:
        raise ValueError(f"value must have the dtype of key ({key.dtype}); got {value.dtype}")
    sd = state[0].dtype
    if state[1].dtype != sd or state[2].dtype != sd:
        raise ValueError("numerator, denominator and log_scale must share one dtype")
    if sd not in (key.dtype, torch.float32):
        raise ValueError(f"the state must be float32 or the key dtype ({key.dtype}); got {sd}")
    c = key.shape[1]
    for name, t in (("time_decay", time_decay), ("time_first", time_first)):
        if t.ndim != 1 or t.shape[0] != c:
            raise ValueError(f"{name} must have shape [C]={c}; got {tuple(t.shape)}")
    if key.dtype not in _CODES:
        raise ValueError(f"unsupported dtype {key.dtype}; expected float32, bfloat16 or float16")


@torch.library.custom_op(
    "spikegpt_b200::wkv_step_",
    mutates_args=("numerator", "denominator", "log_scale"),
    device_types="cuda",
)
def _wkv_step_op(
    key: Tensor,
    value: Tensor,
    time_decay: Tensor,
    time_first: Tensor,
    numerator: Tensor,
    denominator: Tensor,
    log_scale: Tensor,
) -> Tensor:
    y = torch.empty_like(numerator)
    td = time_decay.detach().to(torch.float32).contiguous()
    tf = time_first.detach().to(torch.float32).contiguous()
    b, c = key.shape
    stream = torch.cuda.current_stream(key.device).cuda_stream
    _capi.check(
        _capi.lib().wkv_step(
            _CODES[key.dtype], _CODES[numerator.dtype], key.data_ptr(), value.data_ptr(), td.data_ptr(), tf.data_ptr(),
            numerator.data_ptr(), denominator.data_ptr(), log_scale.data_ptr(), y.data_ptr(), b, c, stream,
        ),
        "wkv_step",
    )
    return y


@_wkv_step_op.register_fake
def _(key, value, time_decay, time_first, numerator, denominator, log_scale):
    return torch.empty_like(numerator)


def weighted_key_value_step_(
    key: Tensor,
    value: Tensor,
    time_decay: Tensor,
    time_first: Tensor,
    numerator: Tensor,
    denominator: Tensor,
    log_scale: Tensor,
) -> Tensor:
    """One WKV step updating (numerator, denominator, log_scale) in place;
    returns the step's WKV output [B, C] in the state's dtype. key and value
    share a dtype; the state is float32 or that dtype (under autocast the
    reference's state is float32 while the projections give bf16 keys, and
    torch promotes the step's result to float32). All [B, C] tensors must be
    contiguous CUDA tensors; time_decay, time_first are [C]."""
    state = (numerator, denominator, log_scale)
    _check(key, value, time_decay, time_first, state)
    if not key.is_cuda:
        raise NotImplementedError("spikegpt_b200.weighted_key_value_step_ runs on CUDA tensors only")
    for name, t in (("key", key), ("value", value), ("numerator", numerator), ("denominator", denominator),
                    ("log_scale", log_scale)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    return torch.ops.spikegpt_b200.wkv_step_(key, value, time_decay, time_first, numerator, denominator, log_scale)


def weighted_key_value_step(
    key: Tensor,
    value: Tensor,
    time_decay: Tensor,
    time_first: Tensor,
    numerator: Tensor,
    denominator: Tensor,
    log_scale: Tensor,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """One WKV step (reference language.py:993-1010) without touching its
    inputs: returns (wkv, numerator, denominator, log_scale), the new state as
    new tensors."""
    state = tuple(t.contiguous().clone() for t in (numerator, denominator, log_scale))
    y = weighted_key_value_step_(key.contiguous(), value.contiguous(), time_decay, time_first, *state)
    return (y, *state)


def initial_step_state(batch_size: int, features: int, *, device, dtype) -> tuple[Tensor, Tensor, Tensor]:
    """(numerator, denominator, log_scale) as the reference's initial_state
    (language.py:957-975): zeros, and the dtype's most negative finite value."""
    z = torch.zeros((batch_size, features), device=device, dtype=dtype)
    return z, z.clone(), torch.full((batch_size, features), torch.finfo(dtype).min, device=device, dtype=dtype)
