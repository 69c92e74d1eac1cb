"""Import the reference's own Python code for tests (and bench.py's CPU legs).

The reference is installed by ``baseline/install_ref.py`` into the git-ignored
``baseline/_ref`` (it travels to GPU boxes with the working tree). Its
dependency ``myelin`` is absent, so the test-only stand-in
``tests/golden/_myelin_shim`` goes on ``sys.path`` first.

``import_language(dropin=True)`` first installs ``spikegpt_b200.dropin`` so the
reference's ``spikegpt.wkv_triton`` / ``spikegpt.wkv_bf16`` imports
(src/spikegpt/language.py:37-38) resolve to this package's ops.
``route_fused_paths(language)`` then makes the CUDA branches of the reference's
model code run: ``has_triton()`` (language.py:1028, 862) reports True, and the
fused LIF entry points it would take from myelin (language.py:867-906:
``myelin.triton.lif_bf16.surrogate_lif_bf16io`` for 16-bit currents,
``triton_surrogate_lif_function`` otherwise; both on time-major [T, B, C]
currents) call this package's LIF op.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
REF_DIR = ROOT / "baseline" / "_ref"
SHIM_DIR = ROOT / "tests" / "golden" / "_myelin_shim"


def available() -> bool:
    return (REF_DIR / "spikegpt" / "language.py").exists()


def _paths() -> None:
    for p in (str(REF_DIR), str(SHIM_DIR)):
        if p not in sys.path:
            sys.path.insert(0, p)


def import_language(*, dropin: bool):
    """The reference's ``spikegpt.language`` module (from baseline/_ref)."""
    if not available():
        raise FileNotFoundError(f"{REF_DIR} has no reference install (run baseline/install_ref.py)")
    _paths()
    if dropin:
        from spikegpt_b200 import dropin as _dropin

        _dropin.install()
    import spikegpt.language as language

    return language


def _lif_time_major(currents, params, slope):
    """Spikes [T, B, C] of this package's LIF op for time-major currents."""
    import spikegpt_b200

    x = currents.movedim(0, 1).contiguous()  # [B, T, C], the op's layout
    spikes = spikegpt_b200.surrogate_lif(x, tau=float(params.tau_mem), threshold=float(params.threshold),
                                         reset=float(params.reset), surrogate_slope=float(slope))
    return spikes.movedim(1, 0)


def route_fused_paths(language) -> None:
    """Make the reference module take its CUDA branches with this package's ops."""
    lif_mod = types.ModuleType("myelin.triton.lif")
    lif_mod.surrogate_id = lambda name: {"atan": 0}[name]
    lif_bf16 = types.ModuleType("myelin.triton.lif_bf16")

    def surrogate_lif_bf16io(currents, initial, params, *, surrogate_slope, surrogate_id):
        if surrogate_id != 0:
            raise NotImplementedError("only the arc-tangent surrogate is routed")
        return _lif_time_major(currents, params, surrogate_slope)

    lif_bf16.surrogate_lif_bf16io = surrogate_lif_bf16io
    pkg = types.ModuleType("myelin.triton")
    pkg.lif, pkg.lif_bf16 = lif_mod, lif_bf16
    sys.modules["myelin.triton"] = pkg
    sys.modules["myelin.triton.lif"] = lif_mod
    sys.modules["myelin.triton.lif_bf16"] = lif_bf16

    def triton_surrogate_lif_function(currents, initial, params, *, surrogate, surrogate_slope, hard_forward):
        if surrogate != "atan" or not hard_forward:
            raise NotImplementedError("only the hard arc-tangent spike is routed")
        return None, _lif_time_major(currents, params, surrogate_slope)

    language.has_triton = lambda: True
    language.triton_surrogate_lif_function = triton_surrogate_lif_function
    language.triton_surrogate_lif_recompute_function = triton_surrogate_lif_function


def unroute(language) -> None:
    """Back to the reference's CPU branches (the stand-in's has_triton is False)."""
    from myelin._optional import has_triton
    from myelin.autograd import triton_surrogate_lif_function, triton_surrogate_lif_recompute_function

    language.has_triton = has_triton
    language.triton_surrogate_lif_function = triton_surrogate_lif_function
    language.triton_surrogate_lif_recompute_function = triton_surrogate_lif_recompute_function
