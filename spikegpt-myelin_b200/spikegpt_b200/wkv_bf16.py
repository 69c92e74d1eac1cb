"""WKV custom ops with native bf16/fp16 I/O: the drop-in for the reference's
``spikegpt.wkv_bf16`` (src/spikegpt/wkv_bf16.py).

Registers ``myelin::wkv_forward_bf16io`` and ``myelin::wkv_backward_bf16io``
with the reference's schemas, fake impls and autograd (wkv_bf16.py:143-215).
k, v and grad_y are read in their own dtype and widened in registers; y,
grad_key and grad_value are written in that dtype; state, checkpoints and the
per-channel gradients stay float32.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _ops

_wkv_forward_bf16io_op = _ops.register("myelin::wkv_forward_bf16io", "myelin::wkv_backward_bf16io")


def weighted_key_value_cuda_bf16io(
    key: Tensor,
    value: Tensor,
    time_decay: Tensor,
    time_first: Tensor,
) -> Tensor:
    """RWKV WKV via the native-dtype-I/O sm_100a custom op (CUDA only)."""
    # with gradients: the state-keeping forward, whose backward skips the
    # forward sweep (eager and torch.compile alike)
    return _ops.call_saving_state(torch.ops.myelin.wkv_forward_bf16io, key, value, time_decay, time_first)


# Drop-in name used by the reference's model code (language.py:37, 1030).
weighted_key_value_triton_bf16io = weighted_key_value_cuda_bf16io
