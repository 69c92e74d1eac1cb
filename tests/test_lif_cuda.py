"""GPU parity of the LIF sequence op (lif_forward / lif_backward through the
registered ops) against the oracle and the reference-generated golden vectors.

Spikes: exactly equal to the float32 oracle on the same (dtype-rounded)
inputs, since the kernels keep the reference step's operation order. Input
gradients: max|x - ref| / max(1, max|ref|) <= 1e-5 (float32 I/O), 2e-2
(bf16/fp16, whose gradients are rounded on store)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch
from _wkvtest import TOL_16BIT, TOL_FP32, scaled_err

from oracle import oracle
from spikegpt_b200 import SpikingSequenceLIF, _capi, surrogate_lif

pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "lif_golden.npz")
CASES = sorted({f.split("/")[0] for f in GOLDEN.files})


def _params(name):
    tau, thr, rst, sl = (float(x) for x in GOLDEN[f"{name}/params"])
    return dict(tau=tau, threshold=thr, reset=rst, surrogate_slope=sl)


def _run(x_np, gs_np, dtype, device, **params):
    x = torch.as_tensor(np.asarray(x_np, np.float32)).to(device=device, dtype=dtype).requires_grad_()
    s = surrogate_lif(x, **params)
    s.backward(torch.as_tensor(np.asarray(gs_np, np.float32)).to(device=device, dtype=dtype))
    return s.detach().double().cpu().numpy(), x.grad.double().cpu().numpy(), x.detach().double().cpu().numpy()


def _oracle(x, gs, **p):
    q = dict(tau=p["tau"], threshold=p["threshold"], reset=p["reset"], slope=p["surrogate_slope"])
    return oracle.lif_forward(x, dtype=np.float32, **q), oracle.lif_backward(gs, x, **q)


@pytest.mark.parametrize("name", CASES)
def test_golden_cases_float32(cuda, name):
    s, gx, _ = _run(GOLDEN[f"{name}/x"], GOLDEN[f"{name}/gs"], torch.float32, cuda, **_params(name))
    np.testing.assert_array_equal(s, GOLDEN[f"{name}/spikes"])
    assert scaled_err(gx, GOLDEN[f"{name}/gx"]) <= TOL_FP32


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("name", CASES)
def test_golden_cases_16bit(cuda, name, dtype):
    p = _params(name)
    s, gx, xr = _run(GOLDEN[f"{name}/x"], GOLDEN[f"{name}/gs"], dtype, cuda, **p)
    gs_r = torch.as_tensor(GOLDEN[f"{name}/gs"]).to(dtype).double().numpy()
    s_ref, gx_ref = _oracle(xr, gs_r, **p)
    np.testing.assert_array_equal(s, s_ref)
    assert scaled_err(gx, gx_ref) <= TOL_16BIT


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_config_shape(cuda, dtype):
    """B=64 T=1024 C=512 (a SpikeGPT-41M block's activation)."""
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((64, 1024, 512)) * 1.5 + 0.3).astype(np.float32)
    gs = rng.standard_normal(x.shape).astype(np.float32)
    s, gx, xr = _run(x, gs, dtype, cuda)
    gs_r = torch.as_tensor(gs).to(dtype).double().numpy()
    s_ref, gx_ref = _oracle(xr, gs_r, tau=2.0, threshold=1.0, reset=0.0, surrogate_slope=2.0)
    np.testing.assert_array_equal(s, s_ref)
    assert scaled_err(gx, gx_ref) <= (TOL_FP32 if dtype == torch.float32 else TOL_16BIT)


@pytest.mark.parametrize("shape", [(2, 17, 70), (3, 1, 64), (1, 33, 8), (2, 40, 130), (1, 16, 64), (2, 64, 66)])
@pytest.mark.parametrize("generic", [False, True])
def test_shapes_tails_and_generic_path(cuda, shape, generic):
    _capi.set_debug_overrides(force_generic=int(generic))
    try:
        rng = np.random.default_rng(sum(shape))
        x = (rng.standard_normal(shape) * 2).astype(np.float32)
        gs = rng.standard_normal(shape).astype(np.float32)
        s, gx, xr = _run(x, gs, torch.float32, cuda)
        s_ref, gx_ref = _oracle(xr, gs, tau=2.0, threshold=1.0, reset=0.0, surrogate_slope=2.0)
        np.testing.assert_array_equal(s, s_ref)
        assert scaled_err(gx, gx_ref) <= TOL_FP32
    finally:
        _capi.set_debug_overrides()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(2, 100, 72), (1, 65, 136), (3, 17, 8), (1, 200, 64), (2, 130, 200)])
def test_tma_path_ragged_tiles_and_channels(cuda, shape, dtype):
    """Aligned rows (TMA path) with a partial last staged tile, a partial last
    sub-tile and a partial last channel block."""
    rng = np.random.default_rng(sum(shape) + 1)
    x = (rng.standard_normal(shape) * 2 + 0.2).astype(np.float32)
    gs = rng.standard_normal(shape).astype(np.float32)
    s, gx, xr = _run(x, gs, dtype, cuda)
    gs_r = torch.as_tensor(gs).to(dtype).double().numpy()
    s_ref, gx_ref = _oracle(xr, gs_r, tau=2.0, threshold=1.0, reset=0.0, surrogate_slope=2.0)
    np.testing.assert_array_equal(s, s_ref)
    assert scaled_err(gx, gx_ref) <= (TOL_FP32 if dtype == torch.float32 else TOL_16BIT)


@pytest.mark.parametrize("generic", [False, True])
def test_non_finite_inputs(cuda, generic):
    """Infinite and NaN currents: a spike on +inf leaves a NaN membrane (the
    reference's v * (1 - s) + reset * s gives inf * 0), which never spikes
    again; -inf and NaN do not spike. Spikes equal the oracle's; gradients
    match it with NaNs in the same places."""
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((2, 40, 64)) * 1.5).astype(np.float32)
    x[0, 3, 5] = np.inf
    x[0, 20, 6] = -np.inf
    x[1, 7, 7] = np.nan
    x[1, 30, 8] = np.inf
    gs = rng.standard_normal(x.shape).astype(np.float32)
    _capi.set_debug_overrides(force_generic=int(generic))
    try:
        s, gx, _ = _run(x, gs, torch.float32, cuda)
    finally:
        _capi.set_debug_overrides(force_generic=0)
    s_ref, gx_ref = _oracle(x, gs, tau=2.0, threshold=1.0, reset=0.0, surrogate_slope=2.0)
    np.testing.assert_array_equal(s, s_ref)
    assert s[0, 4:, 5].sum() == 0 and s[0, 3, 5] == 1
    np.testing.assert_array_equal(np.isnan(gx), np.isnan(gx_ref))
    ok = ~np.isnan(gx_ref)
    assert scaled_err(gx[ok], gx_ref[ok]) <= TOL_FP32


def test_module_contract_and_errors(cuda):
    lif = SpikingSequenceLIF(tau=3.0, threshold=0.5, reset=-0.1, surrogate_slope=4.0)
    assert lif.decay == pytest.approx(1 - 1 / 3)
    x = torch.randn(2, 9, 16, device=cuda)
    out = lif(x)
    assert out.shape == x.shape and out.dtype == x.dtype
    assert set(out.unique().tolist()) <= {0.0, 1.0}
    with pytest.raises(ValueError, match="tau must be positive"):
        SpikingSequenceLIF(tau=0.0)
    with pytest.raises(ValueError, match=r"inputs must have shape \[B, T, C\]"):
        lif(torch.randn(4, 16, device=cuda))
    y = lif(x.double())
    assert y.dtype == torch.float64


def test_no_state_without_grad_and_compile(cuda):
    x = torch.randn(4, 64, 64, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        s0 = surrogate_lif(x)
    fn = torch.compile(lambda t: surrogate_lif(t) * 1.0, fullgraph=True)
    xg = x.clone().requires_grad_()
    s1 = fn(xg)
    assert torch.equal(s0, s1.detach())
    s1.float().sum().backward()
    assert xg.grad is not None and torch.isfinite(xg.grad.float()).all()


def test_lif_kernels_are_counted(cuda):
    before = _capi.launch_counts()
    x = torch.randn(2, 32, 64, device=cuda, requires_grad=True)
    surrogate_lif(x).sum().backward()
    after = _capi.launch_counts()
    assert after["lif_fwd_kernel"] == before["lif_fwd_kernel"] + 1
    assert after["lif_bwd_kernel"] == before["lif_bwd_kernel"] + 1


def _lif_grad(x_np, gs_np, dtype, device, generic=False, segments=0):
    _capi.set_debug_overrides(force_segments=segments, force_generic=int(generic))
    try:
        return _run(x_np, gs_np, dtype, device)
    finally:
        _capi.set_debug_overrides()


@pytest.mark.parametrize("dtype,shape", [(torch.float32, (4, 512, 256)), (torch.bfloat16, (3, 1000, 512)),
                                         (torch.float32, (1, 333, 64))])
def test_segmented_backward(cuda, dtype, shape):
    """Few sequences: the TMA backward splits T into segments (per-segment
    adjoint maps, then all segments at once). The last segment's gradients
    equal the one-sweep generic kernel's bit for bit (same operations from a
    zero adjoint), the earlier ones agree to float32 rounding, and both match
    the oracle."""
    rng = np.random.default_rng(sum(shape) + 7)
    x = (rng.standard_normal(shape) * 1.5 + 0.3).astype(np.float32)
    gs = rng.standard_normal(shape).astype(np.float32)
    s_seg, gx_seg, xr = _lif_grad(x, gs, dtype, cuda)
    s_one, gx_one, _ = _lif_grad(x, gs, dtype, cuda, generic=True)
    np.testing.assert_array_equal(s_seg, s_one)
    rt = 16 if dtype == torch.float32 else 32
    tiles = -(-shape[1] // rt)
    units = -(-(-(-shape[2] // 64)) // 4) * shape[0]
    nseg = min(16, 148 // units, tiles // 2)
    per = -(-tiles // nseg)
    last0 = (-(-tiles // per) - 1) * per * rt  # first step of the last segment
    assert 0 < last0 < shape[1]
    np.testing.assert_array_equal(gx_seg[:, last0:], gx_one[:, last0:])
    tol = TOL_FP32 if dtype == torch.float32 else TOL_16BIT
    assert scaled_err(gx_seg, gx_one) <= tol
    gs_r = torch.as_tensor(gs).to(dtype).double().numpy()
    s_ref, gx_ref = _oracle(xr, gs_r, tau=2.0, threshold=1.0, reset=0.0, surrogate_slope=2.0)
    np.testing.assert_array_equal(s_seg, s_ref)
    assert scaled_err(gx_seg, gx_ref) <= tol


@pytest.mark.parametrize("segments", [2, 3, 7])
def test_forced_segment_counts(cuda, segments):
    shape = (2, 230, 72)  # 15 staged tiles of 16 rows, a ragged last one; 72 channels: a partial block
    rng = np.random.default_rng(segments)
    x = (rng.standard_normal(shape) * 2).astype(np.float32)
    gs = rng.standard_normal(shape).astype(np.float32)
    s, gx, xr = _lif_grad(x, gs, torch.float32, cuda, segments=segments)
    s_ref, gx_ref = _oracle(xr, gs, tau=2.0, threshold=1.0, reset=0.0, surrogate_slope=2.0)
    np.testing.assert_array_equal(s, s_ref)
    assert scaled_err(gx, gx_ref) <= TOL_FP32


def test_segmented_non_finite_inputs(cuda):
    """Non-finite currents in different segments: NaNs of the gradients in the
    oracle's places (a NaN adjoint in a later segment reaches every earlier
    segment through its map, as it does through the sweep)."""
    rng = np.random.default_rng(12)
    x = (rng.standard_normal((2, 128, 64)) * 1.5).astype(np.float32)
    x[0, 3, 5] = np.inf
    x[0, 70, 6] = -np.inf
    x[1, 40, 7] = np.nan
    x[1, 100, 8] = np.inf
    gs = rng.standard_normal(x.shape).astype(np.float32)
    s, gx, _ = _lif_grad(x, gs, torch.float32, cuda, segments=4)
    s_ref, gx_ref = _oracle(x, gs, tau=2.0, threshold=1.0, reset=0.0, surrogate_slope=2.0)
    np.testing.assert_array_equal(s, s_ref)
    np.testing.assert_array_equal(np.isnan(gx), np.isnan(gx_ref))
    ok = ~np.isnan(gx_ref)
    assert scaled_err(gx[ok], gx_ref[ok]) <= TOL_FP32


def _lif_forward_capi(x, segments, tau, threshold=1.0, reset=0.0, slope=2.0):
    """Spikes and checkpoints ([B, ceil(T/16), C] float32, the part of the
    state buffer the forward writes) of lif_forward with the segment count
    forced (1: the sequential forward)."""
    code = {torch.float32: _capi.DTYPE_F32, torch.bfloat16: _capi.DTYPE_BF16}[x.dtype]
    b, t, c = x.shape
    lib = _capi.lib()
    spikes = torch.empty_like(x)
    _capi.set_debug_overrides(force_segments=segments)
    try:
        nbytes = int(lib.lif_state_size(code, b, t, c))  # under the override, as lif_forward checks it
        state = torch.empty(nbytes // 4, dtype=torch.float32, device=x.device)
        _capi.check(lib.lif_forward(code, x.data_ptr(), spikes.data_ptr(), state.data_ptr(), nbytes, b, t, c, tau,
                                    threshold, reset, slope, torch.cuda.current_stream(x.device).cuda_stream),
                    "lif_forward")
        torch.cuda.synchronize()
    finally:
        _capi.set_debug_overrides()
    return spikes, state[:b * (-(-t // 16)) * c].clone()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("case", ["tau2", "tau100", "no_spikes_tau100", "non_finite"])
def test_time_segmented_forward_matches_sequential(cuda, dtype, case):
    """The time-segmented forward (speculated segments, repaired up to the
    first sub-tile boundary where the membranes agree) gives the sequential
    forward's spikes and checkpoints bit for bit: with fast decay (segments
    converge in a sub-tile or two), slow decay and no spikes (segments never
    converge, so the repair runs through every segment in order), and with
    non-finite currents."""
    rng = np.random.default_rng(31)
    shape = (3, 1024, 128)
    x = (rng.standard_normal(shape) * 1.5).astype(np.float32)
    tau = 2.0
    if case in ("tau100", "no_spikes_tau100"):
        tau = 100.0
    if case == "no_spikes_tau100":
        x[:] = 0.0
        x[:, 0] = 0.9  # below threshold: a membrane that decays and never spikes
    if case == "non_finite":
        x[0, 100, 3] = np.inf
        x[1, 300, 5] = np.nan
        x[2, 700, 7] = -np.inf
    xt = torch.as_tensor(x).to(device=cuda, dtype=dtype)
    bits = torch.int16 if dtype == torch.bfloat16 else torch.int32
    s_seq, st_seq = _lif_forward_capi(xt, 1, tau)
    for segments in (0, 3, 8):  # 0: the automatic choice (segmented at tau 2, sequential at tau 100)
        s_seg, st_seg = _lif_forward_capi(xt, segments, tau)
        assert torch.equal(s_seg.view(bits), s_seq.view(bits)), segments
        assert torch.equal(st_seg.view(torch.int32), st_seq.view(torch.int32)), segments
    if tau == 2.0:
        s_ref = oracle.lif_forward(xt.double().cpu().numpy(), dtype=np.float32, tau=tau, threshold=1.0, reset=0.0,
                                   slope=2.0)
        np.testing.assert_array_equal(s_seq.double().cpu().numpy(), s_ref)
