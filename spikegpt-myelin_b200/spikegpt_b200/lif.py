"""LIF sequence op: the spiking activation of SpikeGPT blocks on sm_100a.

The reference's ``SpikingSequenceLIF`` (src/spikegpt/language.py:766-918)
unrolls a leaky integrate-and-fire neuron over ``[B, T, C]`` currents with a
hard spike in the forward pass and a surrogate gradient in the backward pass,
via myelin's fused Triton kernels on CUDA or its per-step loop elsewhere
(language.py:816-843, 907-918). ``surrogate_lif`` is that op as two kernel
launches (forward, backward) of ``libspikegpt_wkv.so``, with the loop's
semantics: per (b, c) over t

    v = v * decay + x_t  (decay = 1 - 1/tau);  s_t = surrogate_slope * (v - threshold) >= 0;
    v = v * (1 - s_t) + reset * s_t

with the membrane in float32 and x, spikes in the input dtype (float64 inputs
run in float32, like the reference's upcast). The backward is the gradient of
that loop with the spike's surrogate derivative
``surrogate_slope / (2 (1 + (pi/2 * centered)^2))``, the published arc-tangent
surrogate (the reference's default ``atan_surrogate``; its exact definition lives
in myelin@68b8ebb, which is not available, so the surrogate is restated rather
than pinned). ``SpikingSequenceLIF`` mirrors the reference module's constructor.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from . import _capi
from ._ops import _CODES


def _state_floats(dtype_code: int, b: int, t: int, c: int) -> int:
    return (int(_capi.lib().lif_state_size(dtype_code, b, t, c)) + 3) // 4


@torch.library.custom_op("spikegpt_b200::lif_forward", mutates_args=(), device_types="cuda")
def _lif_forward_op(
    x: Tensor, tau: float, threshold: float, reset: float, slope: float, save_state: bool
) -> tuple[Tensor, Tensor]:
    b, t, c = x.shape
    code = _CODES[x.dtype]
    spikes = torch.empty_like(x)
    n = _state_floats(code, b, t, c) if save_state else 0
    state = torch.empty(n, dtype=torch.float32, device=x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    _capi.check(
        _capi.lib().lif_forward(code, x.data_ptr(), spikes.data_ptr(), state.data_ptr() if n else None, 4 * n,
                                b, t, c, tau, threshold, reset, slope, stream),
        "lif_forward",
    )
    return spikes, state


@_lif_forward_op.register_fake
def _(x, tau, threshold, reset, slope, save_state):
    n = 0
    if save_state:
        b, t, c = x.shape
        n = b * ((t + 15) // 16) * c
        n = (n * 4 + 255) // 256 * 64
    return torch.empty_like(x), x.new_empty(n, dtype=torch.float32)


@torch.library.custom_op("spikegpt_b200::lif_backward", mutates_args=(), device_types="cuda")
def _lif_backward_op(
    grad_spikes: Tensor, x: Tensor, state: Tensor, tau: float, threshold: float, reset: float, slope: float
) -> Tensor:
    b, t, c = x.shape
    code = _CODES[x.dtype]
    gx = torch.empty_like(x)
    gs = grad_spikes.to(x.dtype).contiguous()
    stream = torch.cuda.current_stream(x.device).cuda_stream
    _capi.check(
        _capi.lib().lif_backward(code, gs.data_ptr(), x.data_ptr(), state.data_ptr(), state.numel() * 4,
                                 gx.data_ptr(), b, t, c, tau, threshold, reset, slope, stream),
        "lif_backward",
    )
    return gx


@_lif_backward_op.register_fake
def _(grad_spikes, x, state, tau, threshold, reset, slope):
    return torch.empty_like(x)


def _setup_context(ctx, inputs, output):
    x, tau, threshold, reset, slope, _save = inputs
    ctx.save_for_backward(x, output[1])
    ctx.params = (tau, threshold, reset, slope)
    ctx.mark_non_differentiable(output[1])


def _backward(ctx, grad_spikes, _grad_state):
    x, state = ctx.saved_tensors
    if state.numel() == 0:
        raise RuntimeError("spikegpt_b200.surrogate_lif: the forward ran without saving its state")
    gx = torch.ops.spikegpt_b200.lif_backward(grad_spikes, x, state, *ctx.params)
    return gx, None, None, None, None, None


_lif_forward_op.register_autograd(_backward, setup_context=_setup_context)


def surrogate_lif(
    inputs: Tensor,
    *,
    tau: float = 2.0,
    threshold: float = 1.0,
    reset: float = 0.0,
    surrogate_slope: float = 2.0,
) -> Tensor:
    """Spikes of the LIF neuron over ``inputs`` [B, T, C] (CUDA), in the input
    dtype; differentiable through the arc-tangent surrogate."""
    if inputs.ndim != 3:
        raise ValueError(f"inputs must have shape [B, T, C]; got {inputs.shape}")
    if tau <= 0.0:
        raise ValueError("tau must be positive")
    if not inputs.is_cuda:
        raise NotImplementedError("spikegpt_b200.surrogate_lif runs on CUDA tensors only")
    orig = inputs.dtype
    x = inputs if orig in _CODES else inputs.float()
    x = x.contiguous()
    save = torch.is_grad_enabled() and x.requires_grad
    spikes, _ = torch.ops.spikegpt_b200.lif_forward(x, float(tau), float(threshold), float(reset),
                                                    float(surrogate_slope), save)
    return spikes.to(orig)


class SpikingSequenceLIF(nn.Module):
    """Drop-in for the reference's ``SpikingSequenceLIF`` (language.py:766-918)
    on CUDA: same constructor and forward contract, the arc-tangent surrogate
    with a hard forward spike (the reference's default configuration)."""

    def __init__(
        self,
        *,
        tau: float = 2.0,
        threshold: float = 1.0,
        reset: float = 0.0,
        surrogate=None,
        surrogate_slope: float = 2.0,
        hard_forward: bool = True,
        fused: bool = True,
        recompute: bool = False,
    ) -> None:
        super().__init__()
        if tau <= 0.0:
            raise ValueError("tau must be positive")
        if not hard_forward:
            raise NotImplementedError("only the hard forward spike (the reference's default) is implemented")
        if surrogate is not None and getattr(surrogate, "__name__", "") != "atan_surrogate":
            raise NotImplementedError("only the arc-tangent surrogate is implemented")
        self.tau = tau
        self.threshold = threshold
        self.reset = reset
        self.surrogate_slope = surrogate_slope
        self.hard_forward = hard_forward
        self.fused = fused
        self.recompute = recompute  # the membrane checkpoints make every backward a recompute

    @property
    def decay(self) -> float:
        return 1.0 - (1.0 / self.tau)

    def forward(self, inputs: Tensor) -> Tensor:
        return surrogate_lif(inputs, tau=self.tau, threshold=self.threshold, reset=self.reset,
                             surrogate_slope=self.surrogate_slope)
