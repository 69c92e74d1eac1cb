"""GPU parity of the RWKV-7 DPLR forward (``spikegpt_b200.rwkv7``) against the
numpy float64 oracle: y and the final state within max|x - ref| /
max(1, max|ref|) <= 1e-5 (float32 arithmetic, sequential like the oracle), on
the benchmark's input distributions, ragged chunk tails, one step, an empty
sequence and a carried initial state; plus the argument checks."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from _wkvtest import TOL_FP32, scaled_err

from oracle import oracle
from spikegpt_b200 import _capi
from spikegpt_b200.rwkv7 import dplr_inputs, rwkv7_forward_op

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,t,h", [(2, 37, 3), (1, 1, 1), (3, 130, 2), (1, 256, 12)])
def test_forward_matches_oracle(cuda, b, t, h):
    ins = dplr_inputs(b, t, h, seed=b * 1000 + t + h)
    y, s = rwkv7_forward_op(*(x.to(cuda) for x in ins))
    y_ref, s_ref = oracle.rwkv7_forward_numpy(*(x.numpy() for x in ins))
    assert scaled_err(y.double().cpu().numpy(), y_ref) <= TOL_FP32
    assert scaled_err(s.double().cpu().numpy(), s_ref) <= TOL_FP32


def test_initial_state_and_chunked_sequence(cuda):
    ins = dplr_inputs(2, 100, 4, seed=3)
    y, s = rwkv7_forward_op(*(x.to(cuda) for x in ins))
    y1, s1 = rwkv7_forward_op(*(x[:, :41].to(cuda) for x in ins))
    y2, s2 = rwkv7_forward_op(*(x[:, 41:].to(cuda) for x in ins), state=s1)
    # the same float32 operations in the same order: equal bit for bit
    assert torch.equal(torch.cat([y1, y2], 1), y)
    assert torch.equal(s2, s)
    _, s_ref = oracle.rwkv7_forward_numpy(*(x.numpy() for x in ins))
    assert scaled_err(s.double().cpu().numpy(), s_ref) <= TOL_FP32


def test_empty_sequence_returns_initial_state(cuda):
    ins = [x.to(cuda) for x in dplr_inputs(2, 0, 3, seed=1)]
    s0 = torch.randn(2, 3, 64, 64, device=cuda)
    y, s = rwkv7_forward_op(*ins, state=s0)
    assert y.shape == (2, 0, 3, 64)
    assert torch.equal(s, s0)


def test_errors_and_launch_count(cuda):
    ins = [x.to(cuda) for x in dplr_inputs(1, 4, 2, seed=2)]
    with pytest.raises(ValueError):
        rwkv7_forward_op(*(x[..., :32] for x in ins))
    with pytest.raises(ValueError):
        rwkv7_forward_op(ins[0].double(), *ins[1:])
    with pytest.raises(ValueError):
        rwkv7_forward_op(*ins, state=torch.zeros(1, 2, 64, 32, device=cuda))
    lib = _capi.lib()
    p = ins[0].data_ptr()
    assert lib.rwkv7_forward(p, p, p, p, p, p, None, p, None, 1, 4, 2, 32, None) == _capi.WKV_ERR_INVALID_ARGUMENT
    assert lib.rwkv7_forward(p + 4, p, p, p, p, p, None, p, None, 1, 4, 2, 64, None) == \
        _capi.WKV_ERR_INVALID_ARGUMENT
    before = _capi.launch_counts()["rwkv7_fwd_kernel"]
    rwkv7_forward_op(*ins)
    assert _capi.launch_counts()["rwkv7_fwd_kernel"] == before + 1
