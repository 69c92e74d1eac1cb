"""The time-segmented LIF forward's algorithm (csrc/lif.cuh,
lif_fwd_seg_kernel: passes A, B, V, C) restated in numpy float32 and checked
against the sequential loop, bit for bit, on the inputs that stress it: fast
decay (segments converge within a sub-tile or two), slow decay and no spikes
(segments never converge, so the in-order repair runs through every segment),
a nonzero reset, and non-finite currents (NaN and infinite membranes never
converge). The kernel itself is checked against the sequential forward and
the oracle on the GPU (tests/test_lif_cuda.py); this pins the algorithm's
exactness on the CPU. The step is the kernel's (language.py:831-841): m = the
membrane times decay, vn = m + x, spike = vn >= threshold (slope >= 1),
m = spike ? reset * decay : vn * decay."""

from __future__ import annotations

import numpy as np
import pytest

KSUB = 16
f32 = np.float32


def _step(m, x, decay, thr, rd):
    vn = (m + x).astype(f32)
    p = vn >= thr
    return np.where(p, rd, (vn * decay).astype(f32)).astype(f32), p


def _sequential(x, decay, thr, rd):
    t, c = x.shape
    s = np.zeros((t, c), bool)
    ck = np.zeros((t // KSUB, c), f32)
    m = np.zeros(c, f32)
    for q in range(t // KSUB):
        ck[q] = m
        for i in range(KSUB):
            m, s[q * KSUB + i] = _step(m, x[q * KSUB + i], decay, thr, rd)
    return s, ck


def _segmented(x, decay, thr, rd, nseg):
    t, c = x.shape
    nt = t // KSUB
    ls = -(-nt // nseg)
    nseg = -(-nt // ls)  # no empty segment
    sb = lambda j: min(nt, j * ls)  # noqa: E731
    s = np.zeros((t, c), bool)
    ck = np.zeros((nt, c), f32)

    def sweep(m, q0, q1, cols):  # writes spikes and checkpoints of columns `cols`
        m = m.copy()
        for q in range(q0, q1):
            ck[q, cols] = m[cols]
            for i in range(KSUB):
                m, sp = _step(m, x[q * KSUB + i], decay, thr, rd)
                s[q * KSUB + i, cols] = sp[cols]
        return m

    everything = slice(None)
    end = [sweep(np.zeros(c, f32), sb(j), sb(j + 1), everything) for j in range(nseg)]  # A

    def converge(j, m0):  # B (and V's reruns): no writes
        q0, n = sb(j), sb(j + 1) - sb(j)
        conv = np.where(m0.view(np.uint32) == ck[q0].view(np.uint32), 0, n)
        m = m0.copy()
        for i in range(n):
            if not (conv == n).any():
                break
            q = q0 + i
            ref = ck[q + 1] if i + 1 < n else end[j]
            for r in range(KSUB):
                m, _ = _step(m, x[q * KSUB + r], decay, thr, rd)
            conv = np.where((conv == n) & (m.view(np.uint32) == ref.view(np.uint32)), i + 1, conv)
        return np.where(conv < n, end[j], m), conv

    eb, cv = {}, {}
    for j in range(1, nseg):
        eb[j], cv[j] = converge(j, end[j - 1])
    start, te, reruns = {}, end[0], 0
    for j in range(1, nseg):  # V
        bad = end[j - 1].view(np.uint32) != te.view(np.uint32)
        start[j] = te.copy()
        conv, e = cv[j], eb[j]
        if bad.any():
            reruns += int(bad.sum())
            e2, c2 = converge(j, te)
            conv, e = np.where(bad, c2, conv), np.where(bad, e2, e)
        cv[j], te = conv, e
    for j in range(1, nseg):  # C: a warp's 64 channels run to the warp's largest point
        for w0 in range(0, c, 64):
            cols = slice(w0, w0 + 64)
            sweep(start[j], sb(j), sb(j) + int(cv[j][cols].max()), cols)
    return s, ck, reruns


def _inputs(case, rng, t, c):
    if case.startswith("no_spikes"):
        x = np.zeros((t, c), f32)
        x[0] = 0.9  # below the threshold: a membrane that only decays
        return x
    x = (rng.standard_normal((t, c)) * 1.5).astype(f32)
    if case == "weak_drive":
        x = (rng.standard_normal((t, c)) * 0.05 + 0.02).astype(f32)
    if case == "non_finite":
        x[40, 3], x[150, 5], x[300, 7] = np.inf, np.nan, -np.inf
    return x


@pytest.mark.parametrize("case,tau,reset", [("normal", 2.0, 0.0), ("normal", 100.0, 0.0),
                                            ("no_spikes", 100.0, 0.0), ("no_spikes", 2.0, 0.0),
                                            ("weak_drive", 50.0, 0.3), ("non_finite", 2.0, 0.0)])
@pytest.mark.parametrize("nseg", [2, 3, 8])
def test_segmented_forward_is_the_sequential_loop(case, tau, reset, nseg):
    rng = np.random.default_rng(7)
    x = _inputs(case, rng, 512, 64)
    decay = f32(1.0 - 1.0 / tau)
    rd = f32(f32(reset) * decay)
    with np.errstate(invalid="ignore", over="ignore"):
        s0, c0 = _sequential(x, decay, f32(1.0), rd)
        s1, c1, reruns = _segmented(x, decay, f32(1.0), rd, nseg)
    np.testing.assert_array_equal(s1, s0)
    np.testing.assert_array_equal(c1.view(np.uint32), c0.view(np.uint32))
    if case == "no_spikes" and tau == 100.0 and nseg > 2:
        assert reruns > 0  # the in-order repair ran
