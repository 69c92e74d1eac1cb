"""Device-side failure path of the copy pipeline (GPU).

Every wait of the time-parallel kernels on a copy barrier is bounded; when it
runs out the kernel sets WKV_DEVERR_PIPELINE_TIMEOUT in the library's sticky
device error flags, waits (bounded) for the copies it did issue, and returns,
so the context stays usable. Here the wait is made to run out without any
fault: the debug hook ``wkv_set_debug_pipeline`` makes every CTA of the forward
skip issuing its first round's copies (a barrier that nothing completes) and
shortens the consumers' wait limit to about a millisecond.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from _wkvtest import TOL_16BIT, config_inputs, scaled_err

from oracle import oracle
from spikegpt_b200 import _capi

pytestmark = pytest.mark.gpu


def test_copy_wait_timeout_is_reported_and_the_context_survives(cuda):
    k, v, td, tf, _ = config_inputs(2, 256, 128, seed=41, kscale=2.0)
    kt, vt = (torch.as_tensor(x).to(cuda, torch.bfloat16) for x in (k, v))
    tdt, tft = torch.as_tensor(td).to(cuda), torch.as_tensor(tf).to(cuda)
    assert _capi.plan(_capi.DTYPE_BF16, 2, 256, 128)[0] == 1  # the TMA (time-parallel) path
    assert _capi.device_error_flags(clear=True) == 0
    _capi.set_debug_overrides(force_segments=1)
    _capi.set_debug_pipeline(wait_limit_cycles=2_000_000, withhold_first_copies=True)
    try:
        torch.ops.myelin.wkv_forward_bf16io(kt, vt, tdt, tft)
        torch.cuda.synchronize()
    finally:
        _capi.set_debug_pipeline()
        _capi.set_debug_overrides()
    assert _capi.device_error_flags(clear=True) == _capi.WKV_DEVERR_PIPELINE_TIMEOUT
    # the same call afterwards runs normally and is right
    y = torch.ops.myelin.wkv_forward_bf16io(kt, vt, tdt, tft)
    torch.cuda.synchronize()
    assert _capi.device_error_flags(clear=True) == 0
    kb = kt.float().cpu().numpy().astype(np.float64)
    vb = vt.float().cpu().numpy().astype(np.float64)
    ref = oracle.forward(kb, vb, td.astype(np.float64), tf.astype(np.float64))
    assert scaled_err(y.float().cpu().numpy(), ref) <= TOL_16BIT


def test_debug_pipeline_rejects_a_negative_limit():
    with pytest.raises(Exception):
        _capi.set_debug_pipeline(wait_limit_cycles=-1)
    _capi.set_debug_pipeline()
