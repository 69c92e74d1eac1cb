"""The CPU oracle is pinned to the reference: every golden vector produced by
the reference's own float64 loop (tests/golden/make_golden.py) must be matched
by both restatements (C and numpy) to float64 rounding."""

from __future__ import annotations

import numpy as np
import pytest
from _wkvtest import golden_inputs, load_golden, scaled_err
from make_golden import CFG0_STRIDE

from oracle import oracle

CASES = load_golden()
NAMES = sorted(CASES)


def test_golden_file_has_every_reference_case():
    expected = {"triton_t1", "triton_t7", "triton_t64", "channels70", "variants_square", "cfg0"}
    expected |= {f"variants_t{t}" for t in (1, 4, 16, 17, 40)}
    assert expected <= set(NAMES)


@pytest.mark.parametrize("name", NAMES)
def test_c_oracle_matches_reference_golden(name):
    k, v, td, tf, gy = golden_inputs(name, CASES)
    y, gk, gv, gtd, gtf = oracle.forward_backward(k, v, td, tf, gy)
    g = CASES[name]
    if name == "cfg0":
        y, gk, gv = (a.reshape(-1)[::CFG0_STRIDE] for a in (y, gk, gv))
    for got, key in zip((y, gk, gv, gtd, gtf), ("y", "gk", "gv", "gtd", "gtf"), strict=True):
        assert scaled_err(got, g[key]) < 1e-12, key


@pytest.mark.parametrize("name", [n for n in NAMES if n != "cfg0"])
def test_numpy_oracle_matches_reference_golden(name):
    k, v, td, tf, gy = golden_inputs(name, CASES)
    y = oracle.forward_numpy(k, v, td, tf)
    gk, gv, gtd, gtf = oracle.backward_numpy(gy, -np.exp(np.asarray(td, np.float64)), tf, k, v)
    g = CASES[name]
    for got, key in zip((y, gk, gv, gtd, gtf), ("y", "gk", "gv", "gtd", "gtf"), strict=True):
        assert scaled_err(got, g[key]) < 1e-12, key


@pytest.mark.parametrize("name", NAMES)
def test_reference_scan_agrees_with_reference_loop(name):
    """The reference's CPU path (associative scan) and its loop agree, so the
    oracle is pinned to both."""
    g = CASES[name]
    if "y_assoc" in g:
        assert scaled_err(g["y_assoc"], g["y"]) < 1e-10
    else:
        assert float(g["y_assoc_maxdiff"][0]) < 1e-10


def test_cfg0_generator_reproduces_fixture_inputs():
    k, v, td, tf, gy = golden_inputs("cfg0")
    sums = [float(np.sum(x, dtype=np.float64)) for x in (k, v, td, tf, gy)]
    np.testing.assert_allclose(sums, CASES["cfg0"]["input_sums"], rtol=0, atol=1e-9)


def test_known_answer_first_step_is_value():
    """y[:, 0] == v[:, 0] (reference tests/test_language.py:31-46)."""
    rng = np.random.default_rng(5)
    k, v = rng.standard_normal((2, 4, 3)), rng.standard_normal((2, 4, 3))
    y = oracle.forward(k, v, np.zeros(3), np.zeros(3))
    np.testing.assert_allclose(y[:, 0], v[:, 0], rtol=1e-15, atol=0)


def test_float32_oracle_tracks_float64():
    k, v, td, tf, gy = golden_inputs("cfg0")
    ref = oracle.forward_backward(k, v, td, tf, gy)
    got = oracle.forward_backward(k, v, td, tf, gy, dtype=np.float32)
    for a, b in zip(got, ref, strict=True):
        assert scaled_err(a, b) < 5e-5


def test_oracle_thread_count_does_not_change_results():
    k, v, td, tf, gy = golden_inputs("triton_t64", CASES)
    one = oracle.forward_backward(k, v, td, tf, gy, threads=1)
    many = oracle.forward_backward(k, v, td, tf, gy, threads=4)
    for a, b in zip(one, many, strict=True):
        np.testing.assert_array_equal(a, b)
