"""CPU: the oracle's recurrent step against golden vectors produced by the
reference's own SpikeTimeMix.step (tests/golden/make_golden_step.py)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
from _wkvtest import scaled_err

from oracle import oracle

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "wkv_step_golden.npz")
SINGLE = ["random_state", "initial_state", "large_keys", "decay_extremes"]


def _case(name):
    return {f.split("/")[1]: GOLDEN[f] for f in GOLDEN.files if f.startswith(name + "/")}


@pytest.mark.parametrize("name", SINGLE)
def test_oracle_step_matches_reference_float64(name):
    g = _case(name)
    got = oracle.step(g["k"], g["v"], g["td"], g["tf"], g["num"], g["den"], g["ls"])
    for field, x in zip(("y", "num", "den", "ls"), got, strict=True):
        assert scaled_err(x, g[f"{field}_f64"]) < 1e-12, field


@pytest.mark.parametrize("name", SINGLE)
def test_oracle_step_float32_tracks_reference_float32(name):
    """The reference evaluates the step in the model dtype; the float32 oracle
    follows the same arithmetic in float32."""
    g = _case(name)
    ls = np.maximum(g["ls"], np.finfo(np.float32).min)
    got = oracle.step(g["k"], g["v"], g["td"], g["tf"], g["num"], g["den"], ls, dtype=np.float32)
    for field, x in zip(("y", "num", "den", "ls"), got, strict=True):
        assert scaled_err(x, g[f"{field}_f32"]) < 1e-6, field


def test_oracle_steps_reproduce_the_reference_sequence():
    g = _case("sequence")
    b, t, c = g["k"].shape
    state = oracle.initial_step_state(b, c)
    ys = []
    for i in range(t):
        y, *state = oracle.step(g["k"][:, i], g["v"][:, i], g["td"], g["tf"], *state)
        ys.append(y)
    ys = np.stack(ys, 1)
    assert scaled_err(ys, g["y_f64"]) < 1e-12
    assert scaled_err(ys, g["y_loop"]) < 1e-12  # the reference's step agrees with its loop oracle
    for field, x in zip(("num", "den", "ls"), state, strict=True):
        assert scaled_err(x, g[f"{field}_f64"]) < 1e-12


def test_first_step_from_initial_state_is_value():
    g = _case("initial_state")
    np.testing.assert_array_equal(g["y_f64"], g["v"].astype(np.float64))
    y, *_ = oracle.step(g["k"], g["v"], g["td"], g["tf"], *oracle.initial_step_state(*g["k"].shape))
    np.testing.assert_array_equal(y, g["v"].astype(np.float64))
