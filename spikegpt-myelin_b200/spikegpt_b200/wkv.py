"""WKV custom ops with float32-I/O semantics: the drop-in for the reference's
``spikegpt.wkv_triton`` (src/spikegpt/wkv_triton.py).

Registers ``myelin::wkv_forward`` and ``myelin::wkv_backward`` with the
reference's schemas, fake impls and autograd (wkv_triton.py:147-218) on top of
the sm_100a kernels of ``libspikegpt_wkv.so``. Any floating dtype is accepted;
the recurrence runs in float32 and y comes back in ``key.dtype``
(wkv_triton.py:152-158). The reference upcasts k/v to float32 copies first; the
kernels here read the native dtype instead, which yields the same float32 values.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _ops

_wkv_forward_op = _ops.register("myelin::wkv_forward", "myelin::wkv_backward")


def weighted_key_value_cuda(
    key: Tensor,
    value: Tensor,
    time_decay: Tensor,
    time_first: Tensor,
) -> Tensor:
    """RWKV WKV recurrence via the sm_100a custom op (CUDA only)."""
    # with gradients: the state-keeping forward, whose backward skips the
    # forward sweep (eager and torch.compile alike)
    return _ops.call_saving_state(torch.ops.myelin.wkv_forward, key, value, time_decay, time_first)


# Drop-in name used by the reference's model code (language.py:37-38, 1032).
weighted_key_value_triton = weighted_key_value_cuda
