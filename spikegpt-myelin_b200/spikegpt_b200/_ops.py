"""Shared host logic of the WKV custom ops: validation, dtype handling,
workspace allocation and the calls through the C ABI.

Both op families (``myelin::wkv_forward``/``wkv_backward`` and their
``_bf16io`` twins) run the same kernels: the library reads float32, bfloat16
and float16 I/O natively and always computes in float32.
"""

from __future__ import annotations

import os

import torch
from torch import Tensor

from . import _capi

_CODES = {
    torch.float32: _capi.DTYPE_F32,
    torch.bfloat16: _capi.DTYPE_BF16,
    torch.float16: _capi.DTYPE_F16,
}


def validate_wkv_inputs(key: Tensor, value: Tensor, time_decay: Tensor, time_first: Tensor) -> None:
    """Shape checks with the messages of the reference's ``_validate_wkv_inputs``
    (src/spikegpt/language.py:379-396), plus the device checks the C ABI needs."""
    if key.shape != value.shape:
        msg = f"key and value must have the same shape; got {key.shape} and {value.shape}"
        raise ValueError(msg)
    if key.ndim != 3:
        msg = f"key and value must have shape [B, T, C]; got {key.shape}"
        raise ValueError(msg)
    if time_decay.shape != (key.shape[-1],):
        msg = f"time_decay must have shape [{key.shape[-1]}]; got {time_decay.shape}"
        raise ValueError(msg)
    if time_first.shape != (key.shape[-1],):
        msg = f"time_first must have shape [{key.shape[-1]}]; got {time_first.shape}"
        raise ValueError(msg)
    _same_cuda_device(key, value, time_decay, time_first)


def _same_cuda_device(*tensors: Tensor) -> None:
    dev = tensors[0].device
    if dev.type != "cuda":
        raise RuntimeError(f"spikegpt_b200 WKV ops need CUDA tensors; got device {dev}")
    for t in tensors[1:]:
        if t.device != dev:
            raise RuntimeError(f"all WKV inputs must be on {dev}; got one on {t.device}")
    for t in tensors:
        if not t.is_floating_point():
            raise TypeError(f"WKV inputs must be floating point; got {t.dtype}")


def _io_dtype(dtype: torch.dtype) -> torch.dtype:
    # float64 (or other) inputs run through the float32 kernels, like the
    # reference's key.float() upcast (wkv_triton.py:154-155).
    return dtype if dtype in _CODES else torch.float32


def _workspace(nbytes: int, device: torch.device) -> tuple[Tensor | None, int]:
    if nbytes == 0:
        return None, 0
    buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
    return buf, buf.data_ptr()


# ---------------------------------------------------------------------------
# Saved forward state (the autograd hand-off)
#
# The reference's backward op takes only (grad_y, w, u, k, v), so on its own it
# must re-run the forward recurrence to recover the state. When gradients are
# needed, the model-facing wrappers (weighted_key_value_triton[_bf16io]) call
# ``spikegpt_b200::wkv_forward_with_state`` instead: the same forward, which
# also returns the recurrence state every 16 steps (float32, 0.75 bytes per
# element of key) as a second output. Its autograd formula hands that state to
# ``spikegpt_b200::wkv_backward_from_state``, which reads key/value once instead
# of twice. Both are traceable custom ops with fake impls, so eager autograd
# and torch.compile graphs (the state becomes a saved activation of the
# compiled forward) take the same path. Calls of the ``myelin::`` ops
# themselves keep the reference's self-contained contract.
# ---------------------------------------------------------------------------

_SAVE_STATE = os.environ.get("SPIKEGPT_WKV_SAVE_STATE", "1") != "0"


def set_state_saving(enabled: bool) -> None:
    """Enable or disable the saved-state hand-off (default: enabled)."""
    global _SAVE_STATE
    _SAVE_STATE = bool(enabled)


def state_saving_enabled() -> bool:
    return _SAVE_STATE


def state_nbytes(b, t, c) -> int:
    """Bytes of the saved forward state (``wkv_state_size`` of the C ABI): float32
    checkpoint rows [B][ceil(T/16)][3][C], then one 32-bit counter per 64-channel
    block, each part rounded up to 256 bytes; at least 16 bytes."""
    ckpt = (b * ((t + 15) // 16) * 3 * c * 4 + 255) // 256 * 256
    counters = (((c + 63) // 64) * 4 + 255) // 256 * 256
    return max(ckpt + counters, 16)


def call_saving_state(op, key: Tensor, value: Tensor, time_decay: Tensor, time_first: Tensor) -> Tensor:
    """y of a forward custom op; when autograd will record the call (grad mode
    on, an input that requires grad), through the state-keeping forward so the
    backward skips the forward sweep."""
    if _SAVE_STATE and torch.is_grad_enabled() and any(
        t.requires_grad for t in (key, value, time_decay, time_first)
    ):
        y, _state = torch.ops.spikegpt_b200.wkv_forward_with_state(key, value, time_decay, time_first)
        return y
    return op(key, value, time_decay, time_first)


def forward(
    key: Tensor, value: Tensor, time_decay: Tensor, time_first: Tensor, *, save_state: bool = False
) -> Tensor | tuple[Tensor, Tensor]:
    """y = WKV(key, value; -exp(time_decay), time_first), y in key.dtype. With
    save_state, also returns the saved state for backward_from_state."""
    validate_wkv_inputs(key, value, time_decay, time_first)
    io = _io_dtype(key.dtype)
    k = key.to(io).contiguous()
    v = value.to(io).contiguous()
    td = time_decay.to(torch.float32).contiguous()
    tf = time_first.to(torch.float32).contiguous()
    b, t, c = k.shape
    y = torch.empty_like(k, memory_format=torch.contiguous_format)
    code = _CODES[io]
    lib = _capi.lib()
    state = None
    with torch.cuda.device(k.device):
        stream = torch.cuda.current_stream(k.device).cuda_stream
        nbytes = int(lib.wkv_forward_workspace_size(code, b, t, c))
        ws, ws_ptr = _workspace(nbytes, k.device)
        if save_state:
            sbytes = state_nbytes(b, t, c)
            if sbytes < int(lib.wkv_state_size(code, b, t, c)):
                raise RuntimeError("spikegpt_b200: state size formula disagrees with wkv_state_size")
            state = torch.empty(sbytes, dtype=torch.uint8, device=k.device)
            rc = lib.wkv_forward_with_state(
                code, k.data_ptr(), v.data_ptr(), td.data_ptr(), tf.data_ptr(), y.data_ptr(),
                state.data_ptr(), state.numel(), b, t, c, ws_ptr, nbytes, stream,
            )
            _capi.check(rc, "wkv_forward_with_state")
        else:
            rc = lib.wkv_forward(
                code, k.data_ptr(), v.data_ptr(), td.data_ptr(), tf.data_ptr(), y.data_ptr(),
                b, t, c, ws_ptr, nbytes, stream,
            )
            _capi.check(rc, "wkv_forward")
    y = y if y.dtype == key.dtype else y.to(key.dtype)
    return (y, state) if save_state else y


def backward(
    grad_y: Tensor, w: Tensor, u: Tensor, k: Tensor, v: Tensor, state: Tensor | None = None, *,
    out: tuple[Tensor, Tensor] | None = None,
) -> list[Tensor]:
    """[grad_key, grad_value, grad_time_decay (already x w), grad_time_first].

    Mirrors the output contract of the reference op (wkv_triton.py:164-198):
    grad_key/grad_value like ``k``, the per-channel grads like ``w``/``u``.
    With ``state`` (from forward(save_state=True) on the same inputs) the
    forward sweep is skipped. ``out`` = (grad_key, grad_value) tensors to
    write into (contiguous, k's shape, k's dtype, which must be a kernel I/O
    dtype); they are the ones returned.
    """
    if k.ndim != 3 or grad_y.shape != k.shape or v.shape != k.shape:
        raise ValueError(
            f"grad_y, k and v must share a [B, T, C] shape; got {grad_y.shape}, {k.shape}, {v.shape}"
        )
    c_dim = k.shape[-1]
    if w.shape != (c_dim,) or u.shape != (c_dim,):
        raise ValueError(f"w and u must have shape [{c_dim}]; got {w.shape} and {u.shape}")
    _same_cuda_device(k, v, grad_y, w, u)
    io = _io_dtype(k.dtype)
    kk = k.to(io).contiguous()
    vv = v.to(io).contiguous()
    gy = grad_y.to(io).contiguous()
    w32 = w.to(torch.float32).contiguous()
    u32 = u.to(torch.float32).contiguous()
    b, t, c = kk.shape
    if out is None:
        gk = torch.empty_like(kk, memory_format=torch.contiguous_format)
        gv = torch.empty_like(kk, memory_format=torch.contiguous_format)
    else:
        gk, gv = out
        for g in (gk, gv):
            if g.shape != kk.shape or g.dtype != io or k.dtype != io or not g.is_contiguous() or g.device != kk.device:
                raise ValueError("out tensors must be contiguous, of k's shape and device, in k's (kernel) dtype")
    gtd = torch.empty(c, dtype=torch.float32, device=kk.device)
    gtf = torch.empty(c, dtype=torch.float32, device=kk.device)
    code = _CODES[io]
    lib = _capi.lib()
    with torch.cuda.device(kk.device):
        stream = torch.cuda.current_stream(kk.device).cuda_stream
        nbytes = int(lib.wkv_backward_workspace_size(code, b, t, c))
        ws, ws_ptr = _workspace(nbytes, kk.device)
        if state is not None:
            if state.device != kk.device or state.dtype != torch.uint8 or not state.is_contiguous():
                raise ValueError("state must be the contiguous uint8 buffer from forward(save_state=True)")
            rc = lib.wkv_backward_from_state(
                code, gy.data_ptr(), w32.data_ptr(), u32.data_ptr(), kk.data_ptr(), vv.data_ptr(),
                state.data_ptr(), state.numel(), gk.data_ptr(), gv.data_ptr(), gtd.data_ptr(),
                gtf.data_ptr(), b, t, c, ws_ptr, nbytes, stream,
            )
            _capi.check(rc, "wkv_backward_from_state")
        else:
            rc = lib.wkv_backward(
                code, gy.data_ptr(), w32.data_ptr(), u32.data_ptr(), kk.data_ptr(), vv.data_ptr(),
                gk.data_ptr(), gv.data_ptr(), gtd.data_ptr(), gtf.data_ptr(),
                b, t, c, ws_ptr, nbytes, stream,
            )
            _capi.check(rc, "wkv_backward")
    out_dtype = k.dtype
    return [gk.to(out_dtype), gv.to(out_dtype), gtd.to(w.dtype), gtf.to(u.dtype)]


def register(namespace_op_fwd: str, namespace_op_bwd: str):
    """Register a forward/backward custom-op pair with the reference's schemas
    (wkv_triton.py:147-218 / wkv_bf16.py:143-215) and its autograd contract.
    Returns the forward op."""

    @torch.library.custom_op(namespace_op_fwd, mutates_args=(), device_types="cuda")
    def wkv_forward_op(key: Tensor, value: Tensor, time_decay: Tensor, time_first: Tensor) -> Tensor:
        return forward(key, value, time_decay, time_first)

    @wkv_forward_op.register_fake
    def _(key, value, time_decay, time_first):
        return torch.empty_like(key)

    @torch.library.custom_op(namespace_op_bwd, mutates_args=(), device_types="cuda")
    def wkv_backward_op(grad_y: Tensor, w: Tensor, u: Tensor, k: Tensor, v: Tensor) -> list[Tensor]:
        return backward(grad_y, w, u, k, v)

    @wkv_backward_op.register_fake
    def _(grad_y, w, u, k, v):
        return [torch.empty_like(k), torch.empty_like(k), torch.empty_like(w), torch.empty_like(u)]

    bwd_name = namespace_op_bwd.split("::")[1]

    def setup_context(ctx, inputs, output):
        ctx.save_for_backward(*inputs)

    def backward_fn(ctx, grad_y):
        key, value, time_decay, time_first = ctx.saved_tensors
        w = -torch.exp(time_decay.float())
        u = time_first.float()
        # The kernels read key/value/grad_y in their own dtype, so the fp32
        # copies the reference glue makes (wkv_triton.py:206-210) are not needed;
        # the float32 results are identical.
        gk, gv, gtd, gtf = getattr(torch.ops.myelin, bwd_name)(grad_y, w, u, key, value)
        return (
            gk.to(key.dtype),
            gv.to(value.dtype),
            gtd.to(time_decay.dtype),
            gtf.to(time_first.dtype),
        )

    wkv_forward_op.register_autograd(backward_fn, setup_context=setup_context)
    return wkv_forward_op


@torch.library.custom_op("spikegpt_b200::wkv_backward_from_state", mutates_args=(), device_types="cuda")
def wkv_backward_from_state_op(
    grad_y: Tensor, w: Tensor, u: Tensor, k: Tensor, v: Tensor, state: Tensor
) -> list[Tensor]:
    """The backward op's contract (wkv_triton.py:164-198) plus the saved state."""
    return backward(grad_y, w, u, k, v, state)


@wkv_backward_from_state_op.register_fake
def _(grad_y, w, u, k, v, state):
    return [torch.empty_like(k), torch.empty_like(k), torch.empty_like(w), torch.empty_like(u)]


@torch.library.custom_op("spikegpt_b200::wkv_forward_with_state", mutates_args=(), device_types="cuda")
def wkv_forward_with_state_op(
    key: Tensor, value: Tensor, time_decay: Tensor, time_first: Tensor
) -> tuple[Tensor, Tensor]:
    """The forward op's contract (wkv_triton.py:147-158) plus the saved state
    (uint8, ``state_nbytes`` long) for ``wkv_backward_from_state``."""
    return forward(key, value, time_decay, time_first, save_state=True)


@wkv_forward_with_state_op.register_fake
def _(key, value, time_decay, time_first):
    b, t, c = key.shape
    return torch.empty_like(key), key.new_empty(state_nbytes(b, t, c), dtype=torch.uint8)


def _with_state_setup_context(ctx, inputs, output):
    ctx.save_for_backward(*inputs, output[1])
    ctx.mark_non_differentiable(output[1])


def _with_state_backward(ctx, grad_y, _grad_state):
    key, value, time_decay, time_first, state = ctx.saved_tensors
    w = -torch.exp(time_decay.float())
    u = time_first.float()
    gk, gv, gtd, gtf = torch.ops.spikegpt_b200.wkv_backward_from_state(grad_y, w, u, key, value, state)
    return gk.to(key.dtype), gv.to(value.dtype), gtd.to(time_decay.dtype), gtf.to(time_first.dtype)


wkv_forward_with_state_op.register_autograd(_with_state_backward, setup_context=_with_state_setup_context)
