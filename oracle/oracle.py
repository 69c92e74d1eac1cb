"""CPU oracle for the WKV recurrence -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module, and only as the checker / the timed CPU
baseline. The shipped library never calls it; the CUDA ops raise when their
extension is missing instead of falling back here.

Two restatements of the reference arithmetic live here:

* ``wkv_oracle.c`` (compiled by :func:`build` into ``oracle/_build``): the
  sequential forward of ``src/spikegpt/language.py:399-449`` and the two-pass
  backward of ``src/spikegpt/wkv_triton.py:60-142``, in float64 and float32,
  threaded over lanes with OpenMP.
* :func:`forward_numpy` / :func:`backward_numpy`: the same two algorithms in
  numpy float64, vectorised over the (b, c) lanes and looping over time.

Parity of both is pinned against golden vectors produced by the reference
itself (``tests/golden/make_golden.py``); see ``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
BUILD_DIR = ORACLE_DIR / "_build"
LIB_PATH = BUILD_DIR / "libwkv_oracle.so"
SOURCE = ORACLE_DIR / "wkv_oracle.c"

_lib: ctypes.CDLL | None = None


def build(force: bool = False) -> Path:
    """Compile ``wkv_oracle.c`` into ``oracle/_build/libwkv_oracle.so`` (gcc + OpenMP)."""
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [
        "gcc",
        "-O2",
        "-fno-fast-math",
        "-ffp-contract=off",
        "-fopenmp",
        "-shared",
        "-fPIC",
        "-std=c11",
        str(SOURCE),
        "-o",
        str(tmp),
        "-lm",
    ]
    subprocess.run(cmd, check=True)
    tmp.replace(LIB_PATH)
    return LIB_PATH


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < SOURCE.stat().st_mtime:
        build()
    lib = ctypes.CDLL(str(LIB_PATH))
    i64, ci, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    for suf in ("f64", "f32"):
        fwd = getattr(lib, f"wkv_oracle_forward_{suf}")
        fwd.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, ci]
        fwd.restype = ci
        bwd = getattr(lib, f"wkv_oracle_backward_{suf}")
        bwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, ci]
        bwd.restype = ci
        stp = getattr(lib, f"wkv_oracle_step_{suf}")
        stp.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i64, i64]
        stp.restype = None
        real = ctypes.c_double if suf == "f64" else ctypes.c_float
        lf = getattr(lib, f"lif_oracle_forward_{suf}")
        lf.argtypes = [vp, vp, i64, i64, i64, real, real, real, real]
        lf.restype = None
        lb = getattr(lib, f"lif_oracle_backward_{suf}")
        lb.argtypes = [vp, vp, vp, i64, i64, i64, real, real, real, real]
        lb.restype = ci
    lib.wkv_oracle_max_threads.restype = ci
    _lib = lib
    return lib


def max_threads() -> int:
    return int(_load().wkv_oracle_max_threads())


def _prep(x: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=dtype)


def _ptr(x: np.ndarray) -> int:
    return x.ctypes.data


def forward(k, v, time_decay, time_first, *, dtype=np.float64, threads: int = 0) -> np.ndarray:
    """y = WKV(k, v; time_decay, time_first). k, v: [B, T, C]; td, tf: [C]."""
    suf = "f64" if np.dtype(dtype) == np.float64 else "f32"
    k, v = _prep(k, dtype), _prep(v, dtype)
    td, tf = _prep(time_decay, dtype), _prep(time_first, dtype)
    b, t, c = k.shape
    y = np.empty_like(k)
    rc = getattr(_load(), f"wkv_oracle_forward_{suf}")(
        _ptr(k), _ptr(v), _ptr(td), _ptr(tf), _ptr(y), b, t, c, threads or max_threads()
    )
    if rc != 0:
        raise RuntimeError(f"wkv oracle forward failed with status {rc}")
    return y


def backward(gy, w, u, k, v, *, dtype=np.float64, threads: int = 0):
    """Returns (gk, gv, g_time_decay, g_time_first) with the reference's contract:
    w = -exp(time_decay) and g_time_decay already includes the *w chain rule."""
    suf = "f64" if np.dtype(dtype) == np.float64 else "f32"
    gy, k, v = _prep(gy, dtype), _prep(k, dtype), _prep(v, dtype)
    w, u = _prep(w, dtype), _prep(u, dtype)
    b, t, c = k.shape
    gk, gv = np.empty_like(k), np.empty_like(k)
    gtd, gtf = np.empty(c, dtype=dtype), np.empty(c, dtype=dtype)
    rc = getattr(_load(), f"wkv_oracle_backward_{suf}")(
        _ptr(gy),
        _ptr(w),
        _ptr(u),
        _ptr(k),
        _ptr(v),
        _ptr(gk),
        _ptr(gv),
        _ptr(gtd),
        _ptr(gtf),
        b,
        t,
        c,
        threads or max_threads(),
    )
    if rc != 0:
        raise RuntimeError(f"wkv oracle backward failed with status {rc}")
    return gk, gv, gtd, gtf


def forward_backward(k, v, time_decay, time_first, gy, *, dtype=np.float64, threads: int = 0):
    """Forward plus backward with w = -exp(time_decay), u = time_first (the
    autograd glue of src/spikegpt/wkv_triton.py:204-216)."""
    td = np.asarray(time_decay, dtype=dtype)
    y = forward(k, v, td, time_first, dtype=dtype, threads=threads)
    w = -np.exp(td)
    grads = backward(gy, w, time_first, k, v, dtype=dtype, threads=threads)
    return (y, *grads)


# ---------------------------------------------------------------------------
# numpy restatement (float64), vectorised over lanes
# ---------------------------------------------------------------------------


def step(k, v, time_decay, time_first, numerator, denominator, log_scale, *, dtype=np.float64):
    """One recurrent step, reference src/spikegpt/language.py:993-1010.

    k, v and the state (numerator, denominator, log_scale; natural-log scale)
    are [B, C]; time_decay, time_first are [C]. Returns (y, numerator,
    denominator, log_scale) as new arrays in ``dtype``.
    """
    suf = "f64" if np.dtype(dtype) == np.float64 else "f32"
    k, v = _prep(k, dtype), _prep(v, dtype)
    td, tf = _prep(time_decay, dtype), _prep(time_first, dtype)
    num, den, ls = (np.array(x, dtype=dtype, copy=True, order="C") for x in (numerator, denominator, log_scale))
    b, c = k.shape
    y = np.empty_like(k)
    getattr(_load(), f"wkv_oracle_step_{suf}")(
        _ptr(k), _ptr(v), _ptr(td), _ptr(tf), _ptr(num), _ptr(den), _ptr(ls), _ptr(y), b, c
    )
    return y, num, den, ls


def initial_step_state(b: int, c: int, dtype=np.float64):
    """The reference's initial state (language.py:964-974): zeros and the
    dtype's most negative finite log_scale."""
    return (np.zeros((b, c), dtype), np.zeros((b, c), dtype), np.full((b, c), np.finfo(dtype).min, dtype))


def lif_forward(x, *, tau=2.0, threshold=1.0, reset=0.0, slope=2.0, dtype=np.float64) -> np.ndarray:
    """Spikes of the LIF sequence op (reference SpikingSequenceLIF,
    src/spikegpt/language.py:766-918) for currents x [B, T, C]."""
    suf = "f64" if np.dtype(dtype) == np.float64 else "f32"
    x = _prep(x, dtype)
    s = np.empty_like(x)
    getattr(_load(), f"lif_oracle_forward_{suf}")(_ptr(x), _ptr(s), *x.shape, tau, threshold, reset, slope)
    return s


def lif_backward(gs, x, *, tau=2.0, threshold=1.0, reset=0.0, slope=2.0, dtype=np.float64) -> np.ndarray:
    """d loss / d x given d loss / d spikes (arc-tangent surrogate; see
    wkv_oracle.c for the formula and why the surrogate is unpinned)."""
    suf = "f64" if np.dtype(dtype) == np.float64 else "f32"
    gs, x = _prep(gs, dtype), _prep(x, dtype)
    gx = np.empty_like(x)
    rc = getattr(_load(), f"lif_oracle_backward_{suf}")(_ptr(gs), _ptr(x), _ptr(gx), *x.shape, tau, threshold,
                                                        reset, slope)
    if rc != 0:
        raise RuntimeError("lif oracle backward failed")
    return gx


def forward_numpy(k, v, time_decay, time_first) -> np.ndarray:
    """language.py:399-449 in numpy float64 (log-scale starts at finfo.min)."""
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    w = -np.exp(np.asarray(time_decay, dtype=np.float64))
    u = np.asarray(time_first, dtype=np.float64)
    b, t, c = k.shape
    num = np.zeros((b, c))
    den = np.zeros((b, c))
    o = np.full((b, c), np.finfo(np.float64).min)
    y = np.empty_like(k)
    with np.errstate(over="ignore", under="ignore"):
        for step in range(t):
            kt, vt = k[:, step], v[:, step]
            no = np.maximum(o, u + kt)
            a, e = np.exp(o - no), np.exp(u + kt - no)
            y[:, step] = (a * num + e * vt) / (a * den + e)
            wo = o + w
            no = np.maximum(wo, kt)
            a, e = np.exp(wo - no), np.exp(kt - no)
            num = a * num + e * vt
            den = a * den + e
            o = no
    return y


def backward_numpy(gy, w, u, k, v):
    """wkv_triton.py:60-142 (+ the sum over b of line 194) in numpy float64."""
    gy = np.asarray(gy, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    w = np.asarray(w, dtype=np.float64)
    u = np.asarray(u, dtype=np.float64)
    b, t, c = k.shape
    ys, zs, zxs = np.empty_like(k), np.empty_like(k), np.empty_like(k)
    p, q, dpdw, dqdw = (np.zeros((b, c)) for _ in range(4))
    o = np.full((b, c), -1e38)
    gw = np.zeros((b, c))
    gu = np.zeros((b, c))
    with np.errstate(over="ignore", under="ignore"):
        for step in range(t):
            kt, vt, gyt = k[:, step], v[:, step], gy[:, step]
            no = np.maximum(o, kt + u)
            a, e = np.exp(o - no), np.exp(kt + u - no)
            iden = 1.0 / (a * q + e)
            yt = (a * p + e * vt) * iden
            ys[:, step], zs[:, step], zxs[:, step] = yt, iden, kt + u - no
            gw += gyt * (dpdw - dqdw * yt) * iden * a
            gu += gyt * (vt - yt) * e * iden
            no = np.maximum(w + o, kt)
            a, e = np.exp(w + o - no), np.exp(kt - no)
            dpdw = a * (p + dpdw)
            dqdw = a * (q + dqdw)
            p = a * p + e * vt
            q = a * q + e
            o = no
        gk, gv = np.empty_like(k), np.empty_like(k)
        gp, gq = np.zeros((b, c)), np.zeros((b, c))
        o = np.full((b, c), -1e38)
        for step in range(t - 1, -1, -1):
            kt, vt, gyt = k[:, step], v[:, step], gy[:, step]
            yt, zt, zxt = ys[:, step], zs[:, step], zxs[:, step]
            a = gyt * zt * np.exp(zxt)
            e = np.exp(kt + o)
            gk[:, step] = a * (vt - yt) + e * (gp * vt + gq)
            gv[:, step] = a + e * gp
            no = np.maximum(w + o, zxt - kt - u)
            a = np.exp(w + o - no)
            e = gyt * zt * np.exp(zxt - kt - u - no)
            gp = a * gp + e
            gq = a * gq - e * yt
            o = no
    return gk, gv, (gw * w).sum(0), gu.sum(0)


def rwkv7_forward_numpy(r, w, k, v, a, b, s0=None):
    """RWKV-7 diagonal-plus-low-rank recurrence in numpy float64 (parity
    unpinned: the reference ships no code for it; this restates the published
    state update). Tensors [B, T, H, N]; per (b, h) with S [N, N] (rows value
    channels, columns key channels):
        S_t = S_{t-1} diag(w_t) + (S_{t-1} a_t) b_t^T + v_t k_t^T,   y_t = S_t r_t.
    Returns (y [B, T, H, N], final state [B, H, N, N])."""
    r, w, k, v, a, b = (np.asarray(x, np.float64) for x in (r, w, k, v, a, b))
    bsz, t, h, n = r.shape
    s = np.zeros((bsz, h, n, n)) if s0 is None else np.array(s0, np.float64)
    y = np.empty_like(r)
    for i in range(t):
        sa = np.einsum("bhij,bhj->bhi", s, a[:, i])
        s = s * w[:, i][:, :, None, :] + sa[..., None] * b[:, i][:, :, None, :] \
            + v[:, i][..., None] * k[:, i][:, :, None, :]
        y[:, i] = np.einsum("bhij,bhj->bhi", s, r[:, i])
    return y, s
