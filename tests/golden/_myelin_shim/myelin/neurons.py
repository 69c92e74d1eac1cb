"""Minimal LIF parameter/state records (never used by the WKV path)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any


@dataclass
class LIFParams:
    tau_mem: Any = 2.0
    threshold: Any = 1.0
    reset: Any = 0.0


@dataclass
class LIFState:
    membrane: Any = None
