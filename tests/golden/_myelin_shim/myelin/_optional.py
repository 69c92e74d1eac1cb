"""``has_triton`` of the test-only myelin stand-in.

False by default, so importing the reference registers no Triton ops (the
golden-vector scripts run its CPU paths). ``MYELIN_SHIM_HAS_TRITON=1`` makes it
True, for a process that runs the reference's own Triton WKV kernels
(src/spikegpt/wkv_triton.py, wkv_bf16.py register them only when it is True)
as the incumbent on a GPU; such a process must not import this package, whose
ops use the same ``myelin::`` names.
"""

import os


def has_triton() -> bool:
    if os.environ.get("MYELIN_SHIM_HAS_TRITON") != "1":
        return False
    try:
        import triton  # noqa: F401
    except ImportError:
        return False
    return True
