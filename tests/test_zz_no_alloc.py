"""GPU test of ``wkv_backward_noalloc``, the backward entry point that allocates
no device memory.

Some hosts of this library must not allocate device memory themselves: their
HBM is owned by another allocator (a framework's caching allocator, a serving
engine's arena), or they reach the library through a thin FFI binding that has
no allocator and cannot manage a workspace's lifetime. ``wkv_backward_noalloc``
serves them by taking its scratch from one static device array inside the
library (``WKV_NOALLOC_SCRATCH_BYTES``, 32 MiB) instead of a caller workspace.

The test calls it through the C ABI twice in a row, on different inputs and
shapes, and checks each result against ``wkv_backward`` (the workspace entry
point) on the same inputs, within the parity tolerances of the other GPU
tests. The array keeps the first call's contents, so the second call also shows
that nothing stale leaks into a later call. The file name sorts last, so a run
that stops at the first failure has run every other test before this one.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch
from _wkvtest import TOL_16BIT, TOL_FP32, config_inputs, scaled_err

from spikegpt_b200 import _capi

pytestmark = pytest.mark.gpu

# Two calls in a row: a segmented plan (small B*C, ragged T) then a sequential
# one (B*C fills the GPU); both fit in the static scratch.
CALLS = [(4, 300, 192, 11), (64, 256, 512, 12)]
DTYPES = {"float32": (torch.float32, _capi.DTYPE_F32, TOL_FP32),
          "bfloat16": (torch.bfloat16, _capi.DTYPE_BF16, TOL_16BIT),
          "float16": (torch.float16, _capi.DTYPE_F16, TOL_16BIT)}


def _inputs(b, t, c, seed, dtype, device):
    k, v, td, tf, gy = config_inputs(b, t, c, seed=seed, kscale=4.0)
    io = [torch.as_tensor(np.asarray(x, np.float32)).to(device=device, dtype=dtype) for x in (gy, k, v)]
    w = (-torch.exp(torch.as_tensor(td, dtype=torch.float64))).float().to(device)
    u = torch.as_tensor(tf, dtype=torch.float32).to(device)
    return io[0], w, u, io[1], io[2]


def _backward(entry, code, gy, w, u, k, v):
    b, t, c = k.shape
    gk = torch.full_like(k, float("nan"))
    gv = torch.full_like(v, float("nan"))
    gtd = torch.full((c,), float("nan"), dtype=torch.float32, device=k.device)
    gtf = torch.full_like(gtd, float("nan"))
    ptrs = [x.data_ptr() for x in (gy, w, u, k, v, gk, gv, gtd, gtf)]
    stream = torch.cuda.current_stream().cuda_stream
    lib = _capi.lib()
    if entry == "noalloc":
        rc = lib.wkv_backward_noalloc(code, *ptrs, b, t, c, stream)
    else:
        size = lib.wkv_backward_workspace_size(code, b, t, c)
        ws = torch.empty(max(size, 1), dtype=torch.uint8, device=k.device)
        rc = lib.wkv_backward(code, *ptrs, b, t, c, ws.data_ptr(), size, stream)
    _capi.check(rc, f"wkv_backward ({entry})")
    torch.cuda.synchronize()
    return [x.double().cpu().numpy() for x in (gk, gv, gtd, gtf)]


@pytest.mark.parametrize("dtype_name", sorted(DTYPES))
def test_noalloc_matches_workspace_backward_on_two_calls(cuda, dtype_name):
    dtype, code, tol = DTYPES[dtype_name]
    _capi.set_debug_overrides()  # default plans, whatever ran before
    for b, t, c, seed in CALLS:
        args = _inputs(b, t, c, seed, dtype, cuda)
        got = _backward("noalloc", code, *args)
        ref = _backward("workspace", code, *args)
        for name, g, r in zip(("grad_key", "grad_value", "grad_time_decay", "grad_time_first"), got, ref,
                              strict=True):
            assert np.isfinite(g).all(), f"{name} not written at B={b} T={t} C={c}"
            err = scaled_err(g, r)
            assert err <= tol, f"{name} at B={b} T={t} C={c}: scaled error {err:.3e} > {tol}"


def test_noalloc_rejects_shapes_beyond_the_static_scratch(cuda):
    b, t, c = 64, 4096, 512  # checkpoints alone need 96 MiB
    lib = _capi.lib()
    null = ctypes.c_void_p(0)
    rc = lib.wkv_backward_noalloc(_capi.DTYPE_BF16, *([null] * 9), b, t, c, null)
    assert rc == _capi.WKV_ERR_INVALID_ARGUMENT
    msg = _capi.last_error()
    assert "scratch" in msg and "wkv_backward" in msg, msg
