"""CPU: the LIF oracle against golden vectors from the reference's own
SpikingSequenceLIF loop under autograd (tests/golden/make_golden_lif.py; the
spike surrogate is the restated arc-tangent one, see that script)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "lif_golden.npz")
CASES = sorted({f.split("/")[0] for f in GOLDEN.files})


def _params(name):
    tau, thr, rst, sl = GOLDEN[f"{name}/params"]
    return dict(tau=tau, threshold=thr, reset=rst, slope=sl)


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_loop(name):
    x, gs = GOLDEN[f"{name}/x"], GOLDEN[f"{name}/gs"]
    np.testing.assert_array_equal(oracle.lif_forward(x, **_params(name)), GOLDEN[f"{name}/spikes"])
    gx = oracle.lif_backward(gs, x, **_params(name))
    assert np.abs(gx - GOLDEN[f"{name}/gx"]).max() < 1e-12


@pytest.mark.parametrize("name", CASES)
def test_float32_oracle_spikes_match_on_these_cases(name):
    """The float32 membrane (the kernels' precision) gives the same spikes here."""
    x = GOLDEN[f"{name}/x"]
    np.testing.assert_array_equal(oracle.lif_forward(x, dtype=np.float32, **_params(name)),
                                  GOLDEN[f"{name}/spikes"])


def test_spikes_are_binary_and_gradients_flow():
    """reference tests/test_language.py:254-263, on the oracle."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 5, 3)) * 2
    s = oracle.lif_forward(x)
    assert set(np.unique(s)) <= {0.0, 1.0}
    gx = oracle.lif_backward(np.ones_like(x), x)
    assert np.isfinite(gx).all() and np.abs(gx).sum() > 0
