"""Surrogate-gradient names so the reference module imports (not used by WKV)."""

from __future__ import annotations

from collections.abc import Callable
from typing import Literal

import torch

SurrogateName = Literal["atan"]
SurrogateFn = Callable[[torch.Tensor], torch.Tensor]
SURROGATE_NAMES: tuple[str, ...] = ("atan",)


def atan_surrogate(x: torch.Tensor) -> torch.Tensor:
    raise RuntimeError("surrogates are not available in this test shim")


def hard_surrogate_spike(x: torch.Tensor, surrogate: SurrogateFn) -> torch.Tensor:
    raise RuntimeError("surrogates are not available in this test shim")


def surrogate_from_name(name: str) -> SurrogateFn:
    return atan_surrogate
