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

import contextlib
import itertools
import threading

import torch
from torch import Tensor

from . import _capi

MAX_MIX = 3


def supported(x: Tensor) -> bool:
    c = x.shape[-1]
    return x.is_cuda and x.dtype == torch.float32 and x.ndim == 3 and c % 128 == 0 and c <= 1024


# The residual connection x + sublayer(ln_shift_mix(x)) gives x two gradient
# contributions that autograd would sum with one more kernel. A sublayer built
# with a residual token instead hands the skip connection's gradient from
# residual_add's backward (which runs first: the sublayer lies between the
# two) to ln_shift_mix's backward, which adds it to grad x inside its kernel.
# That is only sound when both backwards are certain to run in the same
# backward pass, so tokens are handed out only inside ``residual_handoff()``
# (which TrainStep opens around its forward and full ``loss.backward()``),
# outside torch.compile, and for an x that requires grad; everywhere else the
# token is 0 and residual_add returns x's gradient itself.
_RESIDUAL_GRADS: dict[int, Tensor] = {}
# ln_shift_mix backwards run inside residual_handoff() also write bf16(grad x),
# keyed by id(grad x), for the residual_add backward that receives grad x as its
# output gradient (the bf16 spikes' gradient; no separate cast pass). Entries
# nothing takes (an x that is not a residual_add's output) are dropped with
# the handed-over skip gradients.
_BF16_GRADS: dict[int, tuple[Tensor, Tensor]] = {}
_TOKENS = itertools.count(1)
_HANDOFF = threading.local()


@contextlib.contextmanager
def residual_handoff():
    """Allow residual tokens for sublayers built in this thread while the
    context is open. The caller must run one full backward of everything built
    inside, then check ``pending_residual_grads() == 0``."""
    prev = getattr(_HANDOFF, "on", False)
    _HANDOFF.on = True
    try:
        yield
    finally:
        _HANDOFF.on = prev


def new_residual_token(x: Tensor | None = None) -> int:
    """A token pairing one ln_shift_mix with the residual_add that closes its
    sublayer, or 0 (no pairing) outside ``residual_handoff()``, under
    torch.compile, or when ``x`` does not require grad."""
    if not getattr(_HANDOFF, "on", False) or torch.compiler.is_compiling():
        return 0
    if x is not None and not x.requires_grad:
        return 0
    return next(_TOKENS)


def pending_residual_grads() -> int:
    """Handed-over skip gradients that no ln_shift_mix backward has consumed."""
    return len(_RESIDUAL_GRADS)


def drop_residual_grads() -> None:
    _RESIDUAL_GRADS.clear()
    _BF16_GRADS.clear()


@torch.library.custom_op("spikegpt_b200::ln_shift_mix", mutates_args=(), device_types="cuda")
def _ln_shift_mix(x: Tensor, weight: Tensor, bias: Tensor, mix: Tensor, eps: float, token: int) -> list[Tensor]:
    b, t, c = x.shape
    n = mix.shape[0]
    # the n outputs as one [n, B, T, C] tensor: projections that share a shape
    # can then run as one batched GEMM on it
    stacked = torch.empty((n, b, t, c), dtype=torch.bfloat16, device=x.device)
    mean = torch.empty((b, t), dtype=torch.float32, device=x.device)
    rstd = torch.empty_like(mean)
    ptrs = [stacked[i].data_ptr() for i in range(n)] + [None] * (MAX_MIX - n)
    _capi.check(
        _capi.lib().ln_mix_forward(n, x.data_ptr(), weight.data_ptr(), bias.data_ptr(), mix.data_ptr(), *ptrs,
                                   mean.data_ptr(), rstd.data_ptr(), b, t, c, eps,
                                   torch.cuda.current_stream(x.device).cuda_stream),
        "ln_mix_forward",
    )
    return [stacked, mean, rstd]


@_ln_shift_mix.register_fake
def _(x, weight, bias, mix, eps, token):
    b, t, c = x.shape
    return [x.new_empty((mix.shape[0], b, t, c), dtype=torch.bfloat16), x.new_empty((b, t)), x.new_empty((b, t))]


@torch.library.custom_op("spikegpt_b200::ln_shift_mix_backward", mutates_args=(), device_types="cuda")
def _ln_shift_mix_backward(grads: list[Tensor], x: Tensor, weight: Tensor, bias: Tensor, mix: Tensor,
                           mean: Tensor, rstd: Tensor, grad_residual: Tensor | None,
                           bf16_copy: bool = False) -> list[Tensor]:
    """[grad x, grad weight, grad bias, grad mix, bf16(grad x) when ``bf16_copy``
    (else an empty tensor)]."""
    b, t, c = x.shape
    n = mix.shape[0]
    gs = [g.to(torch.bfloat16).contiguous() for g in grads]
    gx = torch.empty_like(x)
    gx16 = torch.empty(x.shape if bf16_copy else (0,), dtype=torch.bfloat16, device=x.device)
    gw = torch.empty_like(weight)
    gb = torch.empty_like(bias)
    gm = torch.empty_like(mix)
    lib = _capi.lib()
    nws = int(lib.ln_mix_workspace_size(n, b, t, c))
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=x.device)
    ptrs = [g.data_ptr() for g in gs] + [None] * (MAX_MIX - n)
    _capi.check(
        lib.ln_mix_backward(n, *ptrs, x.data_ptr(), weight.data_ptr(), bias.data_ptr(), mix.data_ptr(),
                            mean.data_ptr(), rstd.data_ptr(),
                            None if grad_residual is None else grad_residual.data_ptr(), gx.data_ptr(),
                            gx16.data_ptr() if bf16_copy else None, gw.data_ptr(), gb.data_ptr(),
                            gm.data_ptr(), ws.data_ptr(), nws, b, t, c,
                            torch.cuda.current_stream(x.device).cuda_stream),
        "ln_mix_backward",
    )
    return [gx, gw, gb, gm, gx16]


@_ln_shift_mix_backward.register_fake
def _(grads, x, weight, bias, mix, mean, rstd, grad_residual, bf16_copy=False):
    return [torch.empty_like(x), torch.empty_like(weight), torch.empty_like(bias), torch.empty_like(mix),
            x.new_empty(x.shape if bf16_copy else (0,), dtype=torch.bfloat16)]


def _setup(ctx, inputs, output):
    x, weight, bias, mix, _eps, token = inputs
    ctx.save_for_backward(x, weight, bias, mix, output[1], output[2])
    ctx.n = mix.shape[0]
    ctx.token = token
    # inside residual_handoff(): x is normally the residual stream right after
    # a residual_add, whose backward then takes the bf16 copy of grad x
    ctx.bf16_copy = bool(getattr(_HANDOFF, "on", False)) and not torch.compiler.is_compiling()
    ctx.mark_non_differentiable(output[1], output[2])


def _backward(ctx, grads):
    x, weight, bias, mix, mean, rstd = ctx.saved_tensors
    g = grads[0]
    if g is None:
        g = torch.zeros((ctx.n,) + tuple(x.shape), dtype=torch.bfloat16, device=x.device)
    gouts = list(g.unbind(0))
    gres = _RESIDUAL_GRADS.pop(ctx.token, None) if ctx.token else None
    if gres is not None:
        gres = _aligned(gres.float())
    gx, gw, gb, gm, gx16 = torch.ops.spikegpt_b200.ln_shift_mix_backward(gouts, x, weight, bias, mix, mean, rstd,
                                                                         gres, ctx.bf16_copy)
    if ctx.bf16_copy:
        _BF16_GRADS[id(gx)] = (gx, gx16)
    return gx, gw, gb, gm, None, None


_ln_shift_mix.register_autograd(_backward, setup_context=_setup)


def ln_shift_mix_stacked(x: Tensor, weight: Tensor, bias: Tensor, mixes: list[Tensor], eps: float = 1e-5,
                         residual_token: int = 0) -> Tensor:
    """``ln_shift_mix`` with the outputs stacked as one bf16 [len(mixes), B, T, C]
    tensor."""
    if not supported(x):
        raise ValueError("ln_shift_mix needs a contiguous float32 CUDA [B, T, C] tensor with C % 128 == 0, C <= 1024")
    if not 1 <= len(mixes) <= MAX_MIX:
        raise ValueError(f"1..{MAX_MIX} mixing vectors")
    c = x.shape[-1]
    mix = torch.cat([m.reshape(1, c).float() for m in mixes], 0)
    return torch.ops.spikegpt_b200.ln_shift_mix(x.contiguous(), weight.float().contiguous(),
                                                bias.float().contiguous(), mix.contiguous(), float(eps),
                                                int(residual_token))[0]


def ln_shift_mix(x: Tensor, weight: Tensor, bias: Tensor, mixes: list[Tensor], eps: float = 1e-5,
                 residual_token: int = 0) -> list[Tensor]:
    """bf16 ``LayerNorm(x) * m + shift(LayerNorm(x)) * (1 - m)`` for each m in
    ``mixes`` (each [C] or [1, 1, C]); x [B, T, C] float32 CUDA, contiguous.
    ``residual_token`` (from :func:`new_residual_token`) pairs it with the
    ``residual_add(x, ...)`` that closes the sublayer: the skip connection's
    gradient is then added to grad x in this op's backward kernel."""
    return list(ln_shift_mix_stacked(x, weight, bias, mixes, eps, residual_token).unbind(0))


# ------------------------------------------------------------------ gates
#
# The receptance gate ``sigmoid(r) * x`` of time and channel mixing
# (language.py:1022 and 1035, 1195-1196) and the channel-mixing activation
# ``relu(k).square()`` (language.py:1193) on bf16 GEMM outputs, one kernel
# pass forward and one backward each (``gate_*`` and ``relu_square_*`` in the
# C ABI), with the eager bf16 roundings, so the results equal the eager ops'.


def _aligned(t: Tensor) -> Tensor:
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _stream(t: Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


@torch.library.custom_op("spikegpt_b200::gate", mutates_args=(), device_types="cuda")
def _gate(r: Tensor, x: Tensor) -> Tensor:
    out = torch.empty_like(x)
    _capi.check(_capi.lib().gate_forward(r.data_ptr(), x.data_ptr(), out.data_ptr(), x.numel(), _stream(x)),
                "gate_forward")
    return out


@_gate.register_fake
def _(r, x):
    return torch.empty_like(x)


@torch.library.custom_op("spikegpt_b200::gate_backward", mutates_args=(), device_types="cuda")
def _gate_backward(grad: Tensor, r: Tensor, x: Tensor) -> list[Tensor]:
    gr, gx = torch.empty_like(r), torch.empty_like(x)
    _capi.check(_capi.lib().gate_backward(grad.data_ptr(), r.data_ptr(), x.data_ptr(), gr.data_ptr(), gx.data_ptr(),
                                          x.numel(), _stream(x)), "gate_backward")
    return [gr, gx]


@_gate_backward.register_fake
def _(grad, r, x):
    return [torch.empty_like(r), torch.empty_like(x)]


def gate_backward_into(grad: Tensor, r: Tensor, x: Tensor, gr: Tensor, gx: Tensor) -> None:
    """The gate's backward written into ``gr`` and ``gx`` (contiguous bf16 CUDA
    tensors of r's shape): what ``gate``'s autograd computes, for a caller
    that keeps the gradients in buffers of its own (eager use only)."""
    if not gates_supported(r, x, gr, gx) or not (gr.is_contiguous() and gx.is_contiguous()):
        raise ValueError("gate_backward_into needs contiguous bf16 CUDA tensors of one shape")
    grad = _aligned(grad.to(torch.bfloat16))
    r, x = _aligned(r), _aligned(x)
    _capi.check(_capi.lib().gate_backward(grad.data_ptr(), r.data_ptr(), x.data_ptr(), gr.data_ptr(), gx.data_ptr(),
                                          x.numel(), _stream(x)), "gate_backward")


def _gate_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs)


def _gate_grad(ctx, grad):
    r, x = ctx.saved_tensors
    gr, gx = torch.ops.spikegpt_b200.gate_backward(_aligned(grad.to(torch.bfloat16)), r, x)
    return gr, gx


_gate.register_autograd(_gate_grad, setup_context=_gate_setup)


@torch.library.custom_op("spikegpt_b200::relu_square", mutates_args=(), device_types="cuda")
def _relu_square(k: Tensor) -> Tensor:
    out = torch.empty_like(k)
    _capi.check(_capi.lib().relu_square_forward(k.data_ptr(), out.data_ptr(), k.numel(), _stream(k)),
                "relu_square_forward")
    return out


@_relu_square.register_fake
def _(k):
    return torch.empty_like(k)


@torch.library.custom_op("spikegpt_b200::relu_square_backward", mutates_args=(), device_types="cuda")
def _relu_square_backward(grad: Tensor, k: Tensor) -> Tensor:
    gk = torch.empty_like(k)
    _capi.check(_capi.lib().relu_square_backward(grad.data_ptr(), k.data_ptr(), gk.data_ptr(), k.numel(),
                                                 _stream(k)), "relu_square_backward")
    return gk


@_relu_square_backward.register_fake
def _(grad, k):
    return torch.empty_like(k)


def _rsq_setup(ctx, inputs, output):
    ctx.save_for_backward(inputs[0])


def _rsq_grad(ctx, grad):
    (k,) = ctx.saved_tensors
    return torch.ops.spikegpt_b200.relu_square_backward(_aligned(grad.to(torch.bfloat16)), k)


_relu_square.register_autograd(_rsq_grad, setup_context=_rsq_setup)


def gates_supported(*ts: Tensor) -> bool:
    """bf16 CUDA tensors of one shape: what ``gate`` and ``relu_square`` take."""
    return all(t.is_cuda and t.dtype == torch.bfloat16 and t.shape == ts[0].shape for t in ts)


def gate(r: Tensor, x: Tensor) -> Tensor:
    """bf16 ``sigmoid(r) * x`` (the receptance gate), r and x bf16 CUDA tensors
    of one shape."""
    if not gates_supported(r, x):
        raise ValueError("gate needs bf16 CUDA tensors of one shape")
    return torch.ops.spikegpt_b200.gate(_aligned(r), _aligned(x))


def relu_square(k: Tensor) -> Tensor:
    """bf16 ``relu(k) ** 2``, k a bf16 CUDA tensor."""
    if not gates_supported(k):
        raise ValueError("relu_square needs a bf16 CUDA tensor")
    return torch.ops.spikegpt_b200.relu_square(_aligned(k))


# --------------------------------------------------------- residual add
#
# ``residual + lif(sublayer(...))`` (language.py:1353-1358): the float32
# residual stream plus bf16 spikes. PyTorch's type-promoting add takes its
# mixed-dtype (unvectorized) path; ``residual_add_forward`` is one vectorized
# pass with the same values (the bf16 spike converts exactly, one rounded
# add). The backward is the identity for the residual and a cast to bf16 for
# the spikes, as autograd's.


@torch.library.custom_op("spikegpt_b200::residual_add", mutates_args=(), device_types="cuda")
def _residual_add(x: Tensor, spikes: Tensor, token: int) -> Tensor:
    out = torch.empty_like(x)
    _capi.check(_capi.lib().residual_add_forward(x.data_ptr(), spikes.data_ptr(), out.data_ptr(), x.numel(),
                                                 _stream(x)), "residual_add_forward")
    return out


@_residual_add.register_fake
def _(x, spikes, token):
    return torch.empty_like(x)


def _resid_setup(ctx, inputs, output):
    ctx.token = inputs[2]


def _resid_grad(ctx, grad):
    # the spikes' gradient: bf16(grad), already made by the ln_shift_mix
    # backward that produced grad when there is one
    made = _BF16_GRADS.pop(id(grad), None)
    g16 = made[1] if made is not None and made[0] is grad else grad.to(torch.bfloat16)
    if ctx.token:  # the paired ln_shift_mix adds it to grad x in its kernel
        _RESIDUAL_GRADS[ctx.token] = grad
        return None, g16, None
    return grad, g16, None


_residual_add.register_autograd(_resid_grad, setup_context=_resid_setup)


def residual_add(x: Tensor, spikes: Tensor, residual_token: int = 0) -> Tensor:
    """float32 ``x + spikes`` for a float32 x and bf16 spikes of one shape (CUDA).
    With the ``residual_token`` of the ln_shift_mix that reads this x, the
    gradient for x goes to that op's backward instead of a separate sum."""
    if not (x.is_cuda and x.dtype == torch.float32 and spikes.dtype == torch.bfloat16
            and spikes.is_cuda and x.shape == spikes.shape):
        raise ValueError("residual_add needs a float32 x and bf16 spikes of one shape on CUDA")
    return torch.ops.spikegpt_b200.residual_add(_aligned(x), _aligned(spikes), int(residual_token))


# ------------------------------------------------------------ cross-entropy
#
# The language-model loss under bf16 autocast, F.cross_entropy(logits.float(),
# targets) (language.py:1475-1480): a float32 copy of the [rows, V] logits, a
# log-softmax forward and backward, and the gradient cast back to bf16.
# ``cross_entropy_forward`` / ``_backward`` read the bf16 logits in place
# (rows of pitch ld >= V, so a head padded to an aligned width needs no
# slicing copy) and write the bf16 gradient directly. Targets equal to
# PyTorch's ignore_index -100 contribute nothing and the mean divides by the
# count of the others, as PyTorch's does; any other target outside [0, V)
# (which PyTorch rejects) makes the loss NaN and sets the device error flag
# WKV_DEVERR_BAD_TARGET.


@torch.library.custom_op("spikegpt_b200::cross_entropy_rows", mutates_args=(), device_types="cuda")
def _xent(logits: Tensor, targets: Tensor, classes: int) -> list[Tensor]:
    rows, ld = logits.shape
    loss = torch.empty(rows, dtype=torch.float32, device=logits.device)
    lse = torch.empty_like(loss)
    _capi.check(_capi.lib().cross_entropy_forward(logits.data_ptr(), ld, targets.data_ptr(), rows, classes,
                                                  loss.data_ptr(), lse.data_ptr(), _stream(logits)),
                "cross_entropy_forward")
    return [loss, lse]


@_xent.register_fake
def _(logits, targets, classes):
    rows = logits.shape[0]
    return [logits.new_empty(rows, dtype=torch.float32), logits.new_empty(rows, dtype=torch.float32)]


@torch.library.custom_op("spikegpt_b200::cross_entropy_rows_backward", mutates_args=(), device_types="cuda")
def _xent_backward(logits: Tensor, targets: Tensor, lse: Tensor, grad_loss: Tensor, classes: int) -> Tensor:
    rows, ld = logits.shape
    gx = torch.empty_like(logits)
    _capi.check(_capi.lib().cross_entropy_backward(logits.data_ptr(), ld, targets.data_ptr(), lse.data_ptr(),
                                                   grad_loss.data_ptr(), gx.data_ptr(), rows, classes,
                                                   _stream(logits)), "cross_entropy_backward")
    return gx


@_xent_backward.register_fake
def _(logits, targets, lse, grad_loss, classes):
    return torch.empty_like(logits)


def _xent_setup(ctx, inputs, output):
    logits, targets, classes = inputs
    ctx.save_for_backward(logits, targets, output[1])
    ctx.classes = classes
    ctx.mark_non_differentiable(output[1])


def _xent_grad(ctx, grads):
    logits, targets, lse = ctx.saved_tensors
    g = grads[0]
    if g is None:
        g = torch.zeros(logits.shape[0], dtype=torch.float32, device=logits.device)
    gx = torch.ops.spikegpt_b200.cross_entropy_rows_backward(logits, targets, lse, g.float().contiguous(),
                                                             ctx.classes)
    return gx, None, None


_xent.register_autograd(_xent_grad, setup_context=_xent_setup)


def cross_entropy(logits: Tensor, targets: Tensor, classes: int | None = None) -> Tensor:
    """Mean cross-entropy of bf16 logits [rows, ld] (the first ``classes``
    columns are the classes, default all) against int64 targets [rows], with
    PyTorch's ignore_index -100 semantics."""
    if logits.ndim != 2 or logits.dtype != torch.bfloat16 or not logits.is_cuda:
        raise ValueError("cross_entropy takes bf16 CUDA logits [rows, ld]")
    classes = logits.shape[1] if classes is None else int(classes)
    if logits.shape[1] % 8 or not 1 <= classes <= logits.shape[1]:
        raise ValueError("the logits' row pitch must be a multiple of 8 and hold the classes")
    targets = targets.reshape(-1).to(torch.int64).contiguous()
    if targets.numel() != logits.shape[0]:
        raise ValueError("one target per row")
    loss, _ = torch.ops.spikegpt_b200.cross_entropy_rows(_aligned(logits), targets, classes)
    return loss.sum() / (targets != -100).sum()
