"""RWKV-7 diagonal-plus-low-rank (DPLR) time mixing, forward, on sm_100a.

The optional op of the 216M configuration. The reference has no code for it
(its RWKV-7 experiments called an external library, described in
benchmarks/results/optimizer_wkv_experiments_5090.md:34-135), so this is the
published state update, per sequence and head with an N x N state S (rows
value channels, columns key channels):

    S_t = S_{t-1} diag(w_t) + (S_{t-1} a_t) b_t^T + v_t k_t^T,    y_t = S_t r_t

with w_t in (0, 1) the per-key-channel decay and a_t b_t^T the low-rank
(delta-rule) term (RWKV-7 uses a = -kappa_hat, b = kappa_hat * in-context
learning rate). ``rwkv7_forward_op`` calls ``rwkv7_forward`` of
``libspikegpt_wkv.so``: float32 [B, T, H, 64] tensors, an optional initial
state [B, H, 64, 64], and returns y and the final state. Forward only (no
autograd); sequential in T on CUDA cores.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _capi

HEAD_SIZE = 64


@torch.library.custom_op("spikegpt_b200::rwkv7_forward", mutates_args=(), device_types="cuda")
def _rwkv7_forward(r: Tensor, w: Tensor, k: Tensor, v: Tensor, a: Tensor, b: Tensor,
                   state: Tensor | None) -> list[Tensor]:
    bsz, t, h, n = r.shape
    y = torch.empty_like(r)
    s_out = torch.empty((bsz, h, n, n), dtype=torch.float32, device=r.device)
    _capi.check(
        _capi.lib().rwkv7_forward(r.data_ptr(), w.data_ptr(), k.data_ptr(), v.data_ptr(), a.data_ptr(),
                                  b.data_ptr(), None if state is None else state.data_ptr(), y.data_ptr(),
                                  s_out.data_ptr(), bsz, t, h, n, torch.cuda.current_stream(r.device).cuda_stream),
        "rwkv7_forward",
    )
    return [y, s_out]


@_rwkv7_forward.register_fake
def _(r, w, k, v, a, b, state):
    bsz, _, h, n = r.shape
    return [torch.empty_like(r), r.new_empty((bsz, h, n, n))]


def rwkv7_forward_op(r: Tensor, w: Tensor, k: Tensor, v: Tensor, a: Tensor, b: Tensor,
                     state: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """(y, final state) of the DPLR recurrence; all of r, w, k, v, a, b float32
    CUDA [B, T, H, 64] of one shape, state None or [B, H, 64, 64]."""
    ts = (r, w, k, v, a, b)
    if r.ndim != 4 or r.shape[-1] != HEAD_SIZE:
        raise ValueError(f"r must be [B, T, H, {HEAD_SIZE}], got {tuple(r.shape)}")
    if any(x.shape != r.shape for x in ts):
        raise ValueError("r, w, k, v, a, b must have one shape")
    if any(not x.is_cuda or x.dtype != torch.float32 for x in ts):
        raise ValueError("rwkv7_forward_op takes float32 CUDA tensors")
    if state is not None and (state.shape != (r.shape[0], r.shape[2], HEAD_SIZE, HEAD_SIZE)
                              or state.dtype != torch.float32 or not state.is_cuda):
        raise ValueError("state must be float32 CUDA [B, H, 64, 64]")
    y, s = torch.ops.spikegpt_b200.rwkv7_forward(*(x.contiguous() for x in ts),
                                                 None if state is None else state.contiguous())
    return y, s


def dplr_inputs(b: int, t: int, h: int, *, seed: int = 0, device="cpu") -> tuple[Tensor, ...]:
    """Seeded inputs of the op's benchmark configuration: k, v, r ~ N(0, 1);
    decay w = sigmoid(N(0, 1)); kappa ~ N(0, 0.1) normalised per head and step,
    a = -kappa_hat, b = kappa_hat * sigmoid(N(0, 1)) (an in-context learning
    rate in (0, 1), which keeps the state update contractive)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    shape = (b, t, h, HEAD_SIZE)
    r, k, v = (torch.randn(shape, generator=g) for _ in range(3))
    w = torch.sigmoid(torch.randn(shape, generator=g))
    kappa = torch.randn(shape, generator=g) * 0.1
    kh = kappa / kappa.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    lr = torch.sigmoid(torch.randn(shape, generator=g))
    return tuple(x.to(device) for x in (r, w, k, v, -kh, kh * lr))
