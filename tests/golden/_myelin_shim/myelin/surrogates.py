"""Test-only stand-in for myelin.surrogates (myelin@68b8ebb is not installable
offline; the reference imports these names at src/spikegpt/language.py:24-31).

Only what the golden-vector scripts need is defined. ``atan_surrogate`` and
``hard_surrogate_spike`` restate the published arc-tangent surrogate gradient
(SpikingJelly ``surrogate.ATan``; Fang et al., 2021), with the slope applied by
the caller as the reference does (``centered = surrogate_slope * (v - threshold)``,
language.py:834): surrogate(x) = atan(pi/2 * x) / pi + 1/2, whose derivative is
1 / (2 (1 + (pi/2 * x)^2)); the hard spike is the Heaviside step x >= 0 in the
forward pass with that derivative in the backward pass. myelin's own
definitions are not available here, so parity of the LIF surrogate gradient is
unpinned.
"""

from __future__ import annotations

import math
from collections.abc import Callable
from typing import Literal

import torch

SurrogateName = Literal["atan"]
SurrogateFn = Callable[[torch.Tensor], torch.Tensor]
SURROGATE_NAMES: tuple[str, ...] = ("atan",)


def atan_surrogate(x: torch.Tensor) -> torch.Tensor:
    return torch.atan(x * (math.pi / 2)) / math.pi + 0.5


class _HardSpike(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        ctx.save_for_backward(x)
        return (x >= 0).to(x.dtype)

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        return g * (0.5 / (1.0 + (x * (math.pi / 2)) ** 2))


def hard_surrogate_spike(x: torch.Tensor, surrogate: SurrogateFn) -> torch.Tensor:
    if surrogate is not atan_surrogate:
        raise NotImplementedError("the test shim restates only the atan surrogate")
    return _HardSpike.apply(x)


def surrogate_from_name(name: str) -> SurrogateFn:
    return atan_surrogate
