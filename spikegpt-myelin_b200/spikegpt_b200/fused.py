"""Fused LayerNorm + token-shift mixing (the GEMM inputs of the SpikeGPT blocks).

Each time-mixing and channel-mixing sublayer of the reference model
normalises the float32 residual stream and mixes every step with the previous
one, once per projection (src/spikegpt/language.py:344-353 ``_mix_with_previous``,
1009-1012, 1190-1192): ``out_i = h * m_i + h_prev * (1 - m_i)``, ``h =
LayerNorm(x)``, which bf16 autocast then rounds to bf16 for the projection.
Eagerly that is a LayerNorm, a pad and three elementwise passes per output
plus an autocast copy, and about twice that backward (with PyTorch's
LayerNorm weight-gradient reduction). ``ln_shift_mix`` is one kernel pass
forward (``ln_mix_forward``) and one backward (``ln_mix_backward``, whose
parameter gradients are reduced in a fixed order) from ``libspikegpt_wkv.so``.
Float32 x, LayerNorm weight and bias, mixing vectors [n, C] (n <= 3); C a
multiple of 128 up to 1024; outputs bf16.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _capi

MAX_MIX = 3


def supported(x: Tensor) -> bool:
    c = x.shape[-1]
    return x.is_cuda and x.dtype == torch.float32 and x.ndim == 3 and c % 128 == 0 and c <= 1024


@torch.library.custom_op("spikegpt_b200::ln_shift_mix", mutates_args=(), device_types="cuda")
def _ln_shift_mix(x: Tensor, weight: Tensor, bias: Tensor, mix: Tensor, eps: float) -> list[Tensor]:
    b, t, c = x.shape
    n = mix.shape[0]
    outs = [torch.empty((b, t, c), dtype=torch.bfloat16, device=x.device) for _ in range(n)]
    mean = torch.empty((b, t), dtype=torch.float32, device=x.device)
    rstd = torch.empty_like(mean)
    ptrs = [o.data_ptr() for o in outs] + [None] * (MAX_MIX - n)
    _capi.check(
        _capi.lib().ln_mix_forward(n, x.data_ptr(), weight.data_ptr(), bias.data_ptr(), mix.data_ptr(), *ptrs,
                                   mean.data_ptr(), rstd.data_ptr(), b, t, c, eps,
                                   torch.cuda.current_stream(x.device).cuda_stream),
        "ln_mix_forward",
    )
    return outs + [mean, rstd]


@_ln_shift_mix.register_fake
def _(x, weight, bias, mix, eps):
    b, t, c = x.shape
    return [x.new_empty((b, t, c), dtype=torch.bfloat16) for _ in range(mix.shape[0])] + [
        x.new_empty((b, t)), x.new_empty((b, t))]


@torch.library.custom_op("spikegpt_b200::ln_shift_mix_backward", mutates_args=(), device_types="cuda")
def _ln_shift_mix_backward(grads: list[Tensor], x: Tensor, weight: Tensor, bias: Tensor, mix: Tensor,
                           mean: Tensor, rstd: Tensor) -> list[Tensor]:
    b, t, c = x.shape
    n = mix.shape[0]
    gs = [g.to(torch.bfloat16).contiguous() for g in grads]
    gx = torch.empty_like(x)
    gw = torch.empty_like(weight)
    gb = torch.empty_like(bias)
    gm = torch.empty_like(mix)
    lib = _capi.lib()
    nws = int(lib.ln_mix_workspace_size(n, b, t, c))
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=x.device)
    ptrs = [g.data_ptr() for g in gs] + [None] * (MAX_MIX - n)
    _capi.check(
        lib.ln_mix_backward(n, *ptrs, x.data_ptr(), weight.data_ptr(), bias.data_ptr(), mix.data_ptr(),
                            mean.data_ptr(), rstd.data_ptr(), gx.data_ptr(), gw.data_ptr(), gb.data_ptr(),
                            gm.data_ptr(), ws.data_ptr(), nws, b, t, c,
                            torch.cuda.current_stream(x.device).cuda_stream),
        "ln_mix_backward",
    )
    return [gx, gw, gb, gm]


@_ln_shift_mix_backward.register_fake
def _(grads, x, weight, bias, mix, mean, rstd):
    return [torch.empty_like(x), torch.empty_like(weight), torch.empty_like(bias), torch.empty_like(mix)]


def _setup(ctx, inputs, output):
    x, weight, bias, mix, _eps = inputs
    n = mix.shape[0]
    ctx.save_for_backward(x, weight, bias, mix, output[n], output[n + 1])
    ctx.n = n
    ctx.mark_non_differentiable(output[n], output[n + 1])


def _backward(ctx, grads):
    x, weight, bias, mix, mean, rstd = ctx.saved_tensors
    gouts = [g if g is not None else torch.zeros(x.shape, dtype=torch.bfloat16, device=x.device)
             for g in grads[: ctx.n]]
    gx, gw, gb, gm = torch.ops.spikegpt_b200.ln_shift_mix_backward(gouts, x, weight, bias, mix, mean, rstd)
    return gx, gw, gb, gm, None


_ln_shift_mix.register_autograd(_backward, setup_context=_setup)


def ln_shift_mix(x: Tensor, weight: Tensor, bias: Tensor, mixes: list[Tensor], eps: float = 1e-5) -> list[Tensor]:
    """bf16 ``LayerNorm(x) * m + shift(LayerNorm(x)) * (1 - m)`` for each m in
    ``mixes`` (each [C] or [1, 1, C]); x [B, T, C] float32 CUDA, contiguous."""
    if not supported(x):
        raise ValueError("ln_shift_mix needs a contiguous float32 CUDA [B, T, C] tensor with C % 128 == 0, C <= 1024")
    if not 1 <= len(mixes) <= MAX_MIX:
        raise ValueError(f"1..{MAX_MIX} mixing vectors")
    c = x.shape[-1]
    mix = torch.cat([m.reshape(1, c).float() for m in mixes], 0)
    outs = torch.ops.spikegpt_b200.ln_shift_mix(x.contiguous(), weight.float().contiguous(),
                                                bias.float().contiguous(), mix.contiguous(), float(eps))
    return list(outs[: len(mixes)])
