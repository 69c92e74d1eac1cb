"""B200-native (sm_100a) WKV recurrence for SpikeGPT.

Importing the package registers the reference's custom ops
``myelin::wkv_forward``, ``myelin::wkv_backward`` (float32-I/O semantics, module
``spikegpt_b200.wkv``) and ``myelin::wkv_forward_bf16io``,
``myelin::wkv_backward_bf16io`` (native bf16/fp16 I/O, ``spikegpt_b200.wkv_bf16``).
The kernels live in ``libspikegpt_wkv.so`` behind the C ABI of
``include/spikegpt_wkv.h``.
"""

from __future__ import annotations

from . import _capi
from ._ops import set_state_saving, state_saving_enabled, validate_wkv_inputs
from .lif import SpikingSequenceLIF, surrogate_lif
from .step import initial_step_state, weighted_key_value_step, weighted_key_value_step_
from .wkv import weighted_key_value_cuda, weighted_key_value_triton
from .wkv_bf16 import weighted_key_value_cuda_bf16io, weighted_key_value_triton_bf16io

__all__ = [
    "SpikingSequenceLIF",
    "surrogate_lif",
    "initial_step_state",
    "weighted_key_value_step",
    "weighted_key_value_step_",
    "set_state_saving",
    "state_saving_enabled",
    "validate_wkv_inputs",
    "weighted_key_value_cuda",
    "weighted_key_value_cuda_bf16io",
    "weighted_key_value_triton",
    "weighted_key_value_triton_bf16io",
    "_capi",
]
