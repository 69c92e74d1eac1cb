"""Make the reference's model code use these ops without editing it.

``install()`` registers this package's modules under the names the reference
imports them from (``spikegpt.wkv_triton`` and ``spikegpt.wkv_bf16``, imported
at src/spikegpt/language.py:37-38). Call it before ``spikegpt`` is imported.
The reference still gates the CUDA dispatch on ``myelin._optional.has_triton()``
(language.py:1028); that dependency must report True for the op to be used.
"""

from __future__ import annotations

import sys


def install() -> None:
    from . import wkv, wkv_bf16

    for name in ("spikegpt.wkv_triton", "spikegpt.wkv_bf16"):
        loaded = sys.modules.get(name)
        if loaded is not None and loaded not in (wkv, wkv_bf16):
            raise RuntimeError(
                f"{name} is already imported; call spikegpt_b200.dropin.install() before importing spikegpt"
            )
    sys.modules["spikegpt.wkv_triton"] = wkv
    sys.modules["spikegpt.wkv_bf16"] = wkv_bf16
