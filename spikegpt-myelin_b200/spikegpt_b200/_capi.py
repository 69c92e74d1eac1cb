"""ctypes binding of ``libspikegpt_wkv.so`` (C ABI in ``include/spikegpt_wkv.h``).

The library is built in-tree (``spikegpt-myelin_b200/build.py``) into
``spikegpt-myelin_b200/lib/``. There is no fallback: if the library is missing
every op raises, so a silent CPU or eager path can never stand in for it.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_ROOT / "lib" / "libspikegpt_wkv.so"
HEADER_PATH = PKG_ROOT.parent / "include" / "spikegpt_wkv.h"

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
WKV_OK = 0
WKV_ERR_INVALID_ARGUMENT = 1
WKV_ERR_WORKSPACE_TOO_SMALL = 2
WKV_ERR_CUDA = 3
WKV_ERR_DRIVER = 4
WKV_DEVERR_PIPELINE_TIMEOUT = 1
WKV_DEVERR_BAD_TARGET = 2


class WKVError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, status: int, where: str, detail: str) -> None:
        super().__init__(f"{where}: {status_string(status)} (status {status}): {detail}")
        self.status = status


_lib: ctypes.CDLL | None = None
_lock = threading.Lock()


def library_path() -> Path:
    return Path(os.environ.get("SPIKEGPT_WKV_LIB", str(LIB_PATH)))


def lib() -> ctypes.CDLL:
    """Load (once) and return the shared library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"spikegpt_b200: CUDA library {path} is not built; run "
                "`python spikegpt-myelin_b200/build.py` (or __graft_entry__.build())"
            )
        handle = ctypes.CDLL(str(path))
        i64, ci, vp, sz = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t
        handle.wkv_abi_version.argtypes = []
        handle.wkv_abi_version.restype = ci
        handle.wkv_status_string.argtypes = [ci]
        handle.wkv_status_string.restype = ctypes.c_char_p
        handle.wkv_last_error.argtypes = []
        handle.wkv_last_error.restype = ctypes.c_char_p
        handle.wkv_forward_workspace_size.argtypes = [ci, i64, i64, i64]
        handle.wkv_forward_workspace_size.restype = sz
        handle.wkv_backward_workspace_size.argtypes = [ci, i64, i64, i64]
        handle.wkv_backward_workspace_size.restype = sz
        handle.wkv_forward.argtypes = [ci, vp, vp, vp, vp, vp, i64, i64, i64, vp, sz, vp]
        handle.wkv_forward.restype = ci
        handle.wkv_backward.argtypes = [ci, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp, sz, vp]
        handle.wkv_backward.restype = ci
        handle.wkv_backward_noalloc.argtypes = [ci, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp]
        handle.wkv_backward_noalloc.restype = ci
        handle.wkv_step.argtypes = [ci, ci, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, vp]
        handle.wkv_step.restype = ci
        f32 = ctypes.c_float
        handle.lif_state_size.argtypes = [ci, i64, i64, i64]
        handle.lif_state_size.restype = sz
        handle.lif_plan.argtypes = [ci, i64, i64, i64, f32, ci, ctypes.POINTER(ci), ctypes.POINTER(ci)]
        handle.lif_plan.restype = ci
        handle.lif_forward.argtypes = [ci, vp, vp, vp, sz, i64, i64, i64, f32, f32, f32, f32, vp]
        handle.lif_forward.restype = ci
        handle.lif_backward.argtypes = [ci, vp, vp, vp, sz, vp, i64, i64, i64, f32, f32, f32, f32, vp]
        handle.lif_backward.restype = ci
        handle.ln_mix_workspace_size.argtypes = [ci, i64, i64, i64]
        handle.ln_mix_workspace_size.restype = sz
        handle.ln_mix_forward.argtypes = [ci, vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, f32, vp]
        handle.ln_mix_forward.restype = ci
        handle.ln_mix_backward.argtypes = [ci, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                           sz, i64, i64, i64, vp]
        handle.ln_mix_backward.restype = ci
        handle.gate_forward.argtypes = [vp, vp, vp, i64, vp]
        handle.gate_forward.restype = ci
        handle.gate_backward.argtypes = [vp, vp, vp, vp, vp, i64, vp]
        handle.gate_backward.restype = ci
        handle.relu_square_forward.argtypes = [vp, vp, i64, vp]
        handle.relu_square_forward.restype = ci
        handle.relu_square_backward.argtypes = [vp, vp, vp, i64, vp]
        handle.relu_square_backward.restype = ci
        handle.residual_add_forward.argtypes = [vp, vp, vp, i64, vp]
        handle.residual_add_forward.restype = ci
        handle.rwkv7_forward.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, vp]
        handle.rwkv7_forward.restype = ci
        handle.cross_entropy_forward.argtypes = [vp, i64, vp, i64, i64, vp, vp, vp]
        handle.cross_entropy_forward.restype = ci
        handle.cross_entropy_backward.argtypes = [vp, i64, vp, vp, vp, vp, i64, i64, vp]
        handle.cross_entropy_backward.restype = ci
        handle.wkv_state_size.argtypes = [ci, i64, i64, i64]
        handle.wkv_state_size.restype = sz
        handle.wkv_forward_with_state.argtypes = [ci, vp, vp, vp, vp, vp, vp, sz, i64, i64, i64, vp, sz, vp]
        handle.wkv_forward_with_state.restype = ci
        handle.wkv_backward_from_state.argtypes = [
            ci, vp, vp, vp, vp, vp, vp, sz, vp, vp, vp, vp, i64, i64, i64, vp, sz, vp
        ]
        handle.wkv_backward_from_state.restype = ci
        handle.wkv_plan.argtypes = [ci, i64, i64, i64, ctypes.POINTER(ci), ctypes.POINTER(ci)]
        handle.wkv_plan.restype = ci
        handle.wkv_set_debug_pipeline.argtypes = [ctypes.c_longlong, ci]
        handle.wkv_set_debug_pipeline.restype = ci
        handle.wkv_set_debug_overrides.argtypes = [ci, ci, ci]
        handle.wkv_set_debug_overrides.restype = ci
        handle.wkv_kernel_kinds.argtypes = []
        handle.wkv_kernel_kinds.restype = ci
        handle.wkv_kernel_name.argtypes = [ci]
        handle.wkv_kernel_name.restype = ctypes.c_char_p
        handle.wkv_launch_counts.argtypes = [ctypes.POINTER(ctypes.c_longlong), ci]
        handle.wkv_launch_counts.restype = ci
        handle.wkv_timing_enable.argtypes = [ci]
        handle.wkv_timing_enable.restype = ci
        handle.wkv_timing_collect.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong), ci]
        handle.wkv_timing_collect.restype = ci
        handle.wkv_device_error_flags.argtypes = [ctypes.POINTER(ctypes.c_uint), ci]
        handle.wkv_device_error_flags.restype = ci
        _lib = handle
        return handle


def status_string(status: int) -> str:
    try:
        return lib().wkv_status_string(int(status)).decode()
    except Exception:  # pragma: no cover - only while the library is missing
        return "unknown"


def last_error() -> str:
    return lib().wkv_last_error().decode()


def check(status: int, where: str) -> None:
    if status != WKV_OK:
        raise WKVError(status, where, last_error())


def plan(dtype_code: int, b: int, t: int, c: int) -> tuple[bool, int]:
    """(uses TMA, number of time segments) the library picks for a shape."""
    tma, seg = ctypes.c_int(0), ctypes.c_int(0)
    check(lib().wkv_plan(dtype_code, b, t, c, ctypes.byref(tma), ctypes.byref(seg)), "wkv_plan")
    return bool(tma.value), int(seg.value)


def lif_plan(dtype_code: int, b: int, t: int, c: int, tau: float = 2.0, with_state: bool = True) -> tuple[int, int]:
    """(forward segments, backward segments) the LIF op picks for a shape
    (aligned tensors; 1 = the sequential form)."""
    fwd, bwd = ctypes.c_int(0), ctypes.c_int(0)
    check(lib().lif_plan(dtype_code, b, t, c, float(tau), int(with_state), ctypes.byref(fwd), ctypes.byref(bwd)),
          "lif_plan")
    return int(fwd.value), int(bwd.value)


def set_debug_overrides(force_segments: int = 0, force_generic: bool = False, force_slow: bool = False) -> None:
    check(lib().wkv_set_debug_overrides(int(force_segments), int(force_generic), int(force_slow)), "overrides")


def set_debug_pipeline(wait_limit_cycles: int = 0, withhold_first_copies: bool = False) -> None:
    """Failure-path test hook of the forward's copy pipeline (0, False: defaults)."""
    check(lib().wkv_set_debug_pipeline(int(wait_limit_cycles), int(withhold_first_copies)), "wkv_set_debug_pipeline")


def device_error_flags(clear: bool = False) -> int:
    flags = ctypes.c_uint(0)
    check(lib().wkv_device_error_flags(ctypes.byref(flags), int(clear)), "wkv_device_error_flags")
    return int(flags.value)


def kernel_names() -> list[str]:
    n = lib().wkv_kernel_kinds()
    return [lib().wkv_kernel_name(i).decode() for i in range(n)]


def launch_counts() -> dict[str, int]:
    names = kernel_names()
    arr = (ctypes.c_longlong * len(names))()
    check(lib().wkv_launch_counts(arr, len(names)), "wkv_launch_counts")
    return dict(zip(names, (int(x) for x in arr), strict=True))


def timing_enable(on: bool = True) -> None:
    check(lib().wkv_timing_enable(int(on)), "wkv_timing_enable")


def timing_collect() -> dict[str, tuple[float, int]]:
    """{kernel: (summed device ms, timed launches)} since the last collect."""
    names = kernel_names()
    ms = (ctypes.c_double * len(names))()
    n = (ctypes.c_longlong * len(names))()
    check(lib().wkv_timing_collect(ms, n, len(names)), "wkv_timing_collect")
    return {name: (float(ms[i]), int(n[i])) for i, name in enumerate(names)}


def declared_symbols() -> list[str]:
    """Names of the functions declared in include/spikegpt_wkv.h."""
    import re

    text = HEADER_PATH.read_text()
    return sorted(set(re.findall(r"WKV_API\s+[\w\s\*]+?\b((?:wkv|lif|ln_mix|gate|relu_square|residual_add|rwkv7|cross_entropy)_\w+)\s*\(", text)))
