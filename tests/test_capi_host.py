"""The C-ABI library loads and exports every symbol its header declares, and
its host-side argument handling works without a GPU (no compute calls here)."""

from __future__ import annotations

import ctypes
import subprocess

import pytest

from spikegpt_b200 import _capi


def test_library_exports_every_declared_symbol():
    declared = _capi.declared_symbols()
    assert len(declared) >= 10
    lib = _capi.lib()
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(
        ["nm", "-D", "--defined-only", str(_capi.library_path())], capture_output=True, text=True, check=True
    ).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(declared) == exported, "library exports must match include/spikegpt_wkv.h exactly"


def test_abi_version_and_status_strings():
    lib = _capi.lib()
    assert lib.wkv_abi_version() == 1
    assert _capi.status_string(0) == "ok"
    assert "workspace" in _capi.status_string(_capi.WKV_ERR_WORKSPACE_TOO_SMALL)


def test_invalid_arguments_are_rejected_before_any_launch():
    lib = _capi.lib()
    null = ctypes.c_void_p(0)
    rc = lib.wkv_forward(7, null, null, null, null, null, 1, 1, 1, null, 0, null)
    assert rc == _capi.WKV_ERR_INVALID_ARGUMENT and "dtype" in _capi.last_error()
    rc = lib.wkv_forward(0, null, null, null, null, null, -1, 4, 4, null, 0, null)
    assert rc == _capi.WKV_ERR_INVALID_ARGUMENT and "negative" in _capi.last_error()
    rc = lib.wkv_forward(0, null, null, null, null, null, 2, 4, 4, null, 0, null)
    assert rc == _capi.WKV_ERR_INVALID_ARGUMENT and "null" in _capi.last_error()
    rc = lib.wkv_backward(1, null, null, null, null, null, null, null, null, null, 2, 4, 4, null, 0, null)
    assert rc == _capi.WKV_ERR_INVALID_ARGUMENT


def test_empty_forward_is_a_noop():
    lib = _capi.lib()
    null = ctypes.c_void_p(0)
    for b, t, c in ((0, 4, 4), (2, 0, 4), (2, 4, 0)):
        assert lib.wkv_forward(1, null, null, null, null, null, b, t, c, null, 0, null) == 0


def test_workspace_too_small_is_reported():
    lib = _capi.lib()
    need = lib.wkv_backward_workspace_size(1, 4, 64, 64)
    assert need > 0
    fake = ctypes.c_void_p(1 << 20)  # never dereferenced: the size check comes first
    rc = lib.wkv_backward(1, fake, fake, fake, fake, fake, fake, fake, fake, fake, 4, 64, 64, fake, need - 1, None)
    assert rc == _capi.WKV_ERR_WORKSPACE_TOO_SMALL


def test_workspace_sizes_scale_with_the_checkpoint_grid():
    lib = _capi.lib()
    # sequential plan: checkpoints (3 floats per lane per 16 steps) + partials
    b, t, c = 64, 1024, 512
    ws = lib.wkv_backward_workspace_size(1, b, t, c)
    assert ws >= b * (t // 16) * 3 * c * 4
    assert ws < b * t * c * 2 // 2  # under half of one bf16 [B,T,C] tensor
    assert lib.wkv_forward_workspace_size(1, b, t, c) == 0


@pytest.mark.parametrize(
    "dtype,b,t,c,tma",
    [(1, 64, 1024, 512, True), (0, 64, 1024, 512, True), (1, 3, 7, 70, False), (0, 2, 16, 70, False),
     (1, 2, 16, 40, True), (0, 2, 16, 36, True), (2, 1, 64, 8, True)],
)
def test_plan_tma_eligibility(dtype, b, t, c, tma):
    got_tma, seg = _capi.plan(dtype, b, t, c)
    assert got_tma == tma
    assert seg >= 1


def test_plan_splits_time_when_lanes_are_few():
    _, seg_big = _capi.plan(1, 64, 1024, 512)
    _, seg_small = _capi.plan(1, 1, 3072, 512)
    assert seg_big == 1
    assert seg_small > 1


def test_debug_overrides_change_the_plan_and_reset():
    try:
        _capi.set_debug_overrides(force_segments=3, force_generic=True)
        tma, seg = _capi.plan(1, 64, 1024, 512)
        assert (tma, seg) == (False, 3)
    finally:
        _capi.set_debug_overrides()
    assert _capi.plan(1, 64, 1024, 512) == (True, 1)


@pytest.mark.parametrize("b,t,nseg", [(64, 1024, 1), (24, 1024, 1), (12, 1024, 6), (8, 1024, 8), (4, 1024, 8),
                                      (1, 1024, 8), (24, 3072, 3), (12, 3072, 6), (8, 3072, 8), (4, 3072, 16),
                                      (1, 3072, 16)])
def test_plan_follows_the_measured_segment_choice(b, t, nseg):
    """The segment counts the plan picks on a 148-SM device (the host fallback
    here) at the swept shapes (C = 512, bf16)."""
    assert _capi.plan(1, b, t, 512) == (True, nseg)


def test_lif_plan_segments_the_forward_for_few_sequences():
    """The LIF forward runs time-segmented only with few (64-channel block,
    row) units, T a multiple of 16, C a multiple of 64, the checkpoints
    requested and tau <= 4; it stays sequential at 64 sequences of 512
    channels (the one-GPU SpikeGPT-41M step)."""
    bf16, f32 = _capi.DTYPE_BF16, _capi.DTYPE_F32
    assert _capi.lif_plan(bf16, 64, 1024, 512)[0] == 1
    assert _capi.lif_plan(bf16, 8, 1024, 512)[0] == 8  # the 8-GPU share of global batch 64
    assert _capi.lif_plan(bf16, 32, 1024, 512)[0] == 8  # 256 units: the largest segmented case
    assert _capi.lif_plan(bf16, 33, 1024, 512)[0] == 1
    assert _capi.lif_plan(f32, 4, 512, 256)[0] == 8
    assert _capi.lif_plan(bf16, 8, 1000, 512)[0] == 1  # T not a multiple of 16
    assert _capi.lif_plan(bf16, 8, 1024, 72)[0] == 1  # a partial channel block
    assert _capi.lif_plan(bf16, 8, 1024, 512, tau=100.0)[0] == 1  # slow decay
    assert _capi.lif_plan(bf16, 8, 1024, 512, with_state=False)[0] == 1  # no checkpoints (no grad)
    assert _capi.lif_plan(bf16, 8, 48, 512)[0] == 1  # under 4 sub-tiles a segment
    _capi.set_debug_overrides(force_segments=3)
    try:
        assert _capi.lif_plan(bf16, 64, 1024, 512)[0] == 3
        assert _capi.lif_plan(bf16, 8, 1024, 512, tau=100.0)[0] == 3
    finally:
        _capi.set_debug_overrides()
    with pytest.raises(_capi.WKVError):
        _capi.lif_plan(bf16, 8, 1024, 512, tau=0.0)
