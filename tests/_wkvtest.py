"""Helpers shared by the WKV tests (golden fixtures, tolerances, oracle calls)."""

from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden" / "wkv_golden.npz"

# Tolerances of the parity contract: max|x - ref| / max(1, max|ref|).
TOL_FP32 = 1e-5
TOL_16BIT = 2e-2


def scaled_err(x, ref) -> float:
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if ref.size == 0:
        return 0.0
    return float(np.abs(x - ref).max() / max(1.0, float(np.abs(ref).max())))


def load_golden() -> dict[str, dict[str, np.ndarray]]:
    data = np.load(GOLDEN)
    cases: dict[str, dict[str, np.ndarray]] = {}
    for key in data.files:
        case, field = key.split("/")
        cases.setdefault(case, {})[field] = data[key]
    return cases


def golden_inputs(case: str, cases=None):
    """(k, v, td, tf, gy) of a golden case; cfg0 inputs are regenerated from seed."""
    from make_golden import cfg0_inputs

    if case == "cfg0":
        return cfg0_inputs()
    cases = cases or load_golden()
    c = cases[case]
    return c["k"], c["v"], c["td"], c["tf"], c["gy"]


def config_inputs(b: int, t: int, c: int, *, seed: int = 0, kscale: float = 1.0):
    """Benchmark-config distributions: k, v ~ N(0,1)*kscale; td ~ U(-5,1); tf ~
    U(-1,1); gy ~ N(0,1) (float32, numpy PCG64)."""
    from make_golden import cfg0_inputs

    return cfg0_inputs(b, t, c, seed=seed, kscale=kscale)
