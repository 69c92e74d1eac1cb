"""SpikeGPT language model on this package's sm_100a ops (the train-step harness).

The architecture of the reference's ``SpikeLanguageModel``
(src/spikegpt/language.py:1361-1480) with its defaults (``model_type="rwkv"``,
``attention="rwkv"``, ``spiking=True``, ``spike_embedding=True``,
``spike_input=False``): a spiking token embedding, ``n_layer`` blocks of
RWKV-4 time mixing and channel mixing each followed by a LIF activation on the
residual branch, a final LayerNorm and a linear head. The WKV recurrence runs
on ``weighted_key_value_cuda_bf16io`` / ``weighted_key_value_cuda`` and the LIF
activations on ``surrogate_lif``; everything else is plain PyTorch (cuBLAS
GEMMs under bf16 autocast). Parameter shapes and initial values follow the
reference (language.py:920-955 time mixing, 1145-1160 channel mixing,
1223-1270 block, 1364-1385 model and weight init), so the parameter count of
the SpikeGPT-41M configuration (12 layers, 512 wide, vocabulary 256, context
1024) is the reference's 41,226,240.

The model needs CUDA tensors for its forward pass (the ops have no CPU path);
building it on the CPU is fine.
"""

from __future__ import annotations

import contextlib
import os

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import _ops, fused
from .lif import surrogate_lif
from .wkv import weighted_key_value_cuda
from .wkv_bf16 import weighted_key_value_cuda_bf16io


@dataclass
class SpikeGPTConfig:
    """The reference's SpikeGPTConfig fields this model implements
    (language.py:234-253)."""

    vocab_size: int = 256
    context_length: int = 1024
    n_layer: int = 12
    n_embd: int = 512
    dropout: float = 0.0
    lif_tau: float = 2.0
    lif_threshold: float = 1.0
    lif_reset: float = 0.0
    surrogate_slope: float = 2.0
    spike_embedding: bool = True

    def validate(self) -> None:
        for name in ("vocab_size", "context_length", "n_layer", "n_embd"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if not 0.0 <= self.dropout < 1.0:
            raise ValueError("dropout must be in [0, 1)")
        if self.lif_tau <= 0.0:
            raise ValueError("lif_tau must be positive")


SPIKEGPT_41M = SpikeGPTConfig(vocab_size=256, context_length=1024, n_layer=12, n_embd=512)
# The 216M-class configuration: 18 layers, 768 wide, the GPT-2 BPE vocabulary.
SPIKEGPT_216M = SpikeGPTConfig(vocab_size=50257, context_length=1024, n_layer=18, n_embd=768)


class _HardSpike(torch.autograd.Function):
    """Heaviside spike of ``x`` with the arc-tangent surrogate gradient
    ``1 / (2 (1 + (pi/2 x)^2))``: the spiking embedding's activation (reference
    ``hard_surrogate_spike(slope * e, atan_surrogate)``, language.py:1387-1395)."""

    @staticmethod
    def forward(ctx, x: Tensor) -> Tensor:
        ctx.save_for_backward(x)
        return (x >= 0).to(x.dtype)

    @staticmethod
    def backward(ctx, grad: Tensor) -> Tensor:
        (x,) = ctx.saved_tensors
        h = x * (math.pi / 2)
        return grad * (0.5 / (1.0 + h * h))


def _shift_mix(x: Tensor, mix: Tensor) -> Tensor:
    """``x * mix + x_{t-1} * (1 - mix)`` with a zero row before t = 0
    (reference _mix_with_previous, language.py:344-353)."""
    prev = F.pad(x[:, :-1], (0, 0, 1, 0))
    return x * mix + prev * (1.0 - mix)


def _mix_profile(n_embd: int, power: float, offset: float = 0.0) -> Tensor:
    position = torch.arange(n_embd, dtype=torch.float32) / n_embd
    return (torch.pow(position, power) + offset).view(1, 1, -1)


# The time-mixing key, value and receptance projections as one batched GEMM
# (SPIKEGPT_BATCHED_KVR=0: three GEMMs).
# ------------------------------------------------------------- weight cache
#
# Under bf16 autocast every projection casts its float32 weight to bf16 in the
# forward and widens its bf16 weight gradient back to float32 in the backward:
# two small kernels per weight and step, about 200 in SpikeGPT-41M, which at a
# few sequences per GPU cost as much as the LIF recurrences. A train step can
# instead cast all matmul weights with one kernel and hand the projections
# their bf16 copies: inside ``weight_cache(entries)`` a projection whose weight
# has an entry (bf16 copy, bf16 gradient buffer) multiplies by the copy, and its
# backward writes the bf16 weight gradient into the buffer instead of handing
# the parameter a gradient through autograd; the caller widens the buffers
# into the float32 gradients with one kernel. The values are autocast's: the
# copy is the round-to-nearest cast, and the weight gradient is the same bf16
# product, widened exactly. The key, value and receptance weights of a time
# mixing have one more entry under the tuple of their ids: the [3, C, C] copy
# and gradient buffer of the three, for the batched projection.
#
# With a side stream, each weight-gradient product runs there (forked from the
# backward's stream when its operands are ready): nothing in the backward reads
# it, so it overlaps the rest of the backward, whose kernels leave most SMs idle
# at a few sequences per GPU. The caller joins the side stream before reading
# the gradient buffers, and until then ``side_operands()`` holds the products'
# operands, so the caching allocator (and a graph capture's memory pool) cannot
# hand their memory out while a product still reads it.

_CACHE: dict = {}
_SIDE: list = [None]  # the weight-gradient stream while a cache is active
_SIDE_KEEP: list = []  # operands of the products issued on it since the last join


@contextlib.contextmanager
def weight_cache(entries: dict, side_stream=None):
    """Projections read their weights' bf16 copies from ``entries`` (id of the
    parameter -> (bf16 copy, bf16 gradient buffer)) inside the block; weight
    gradients go to ``side_stream`` when one is given. The cache is state of
    this module: one block at a time per process (not nested, not from two
    threads at once); TrainStep enters it around each forward it issues."""
    _CACHE.update(entries)
    _SIDE[0] = side_stream
    try:
        yield
    finally:
        _CACHE.clear()
        _SIDE[0] = None


def side_operands() -> list:
    """The operands of the weight-gradient products issued on the side stream
    since the caller last cleared this list (after joining the stream)."""
    return _SIDE_KEEP


def _weight_grad(side, product, *operands: Tensor) -> None:
    """Run ``product()`` (which writes a weight gradient buffer) on the side
    stream after the current stream's work so far, or inline without one."""
    if side is None:
        product()
        return
    side.wait_stream(torch.cuda.current_stream(operands[0].device))
    with torch.cuda.stream(side):
        product()
    _SIDE_KEEP.extend(operands)


class _CachedLinear(torch.autograd.Function):
    """``x @ wb.T`` with a cached bf16 weight; the backward returns grad x and
    writes grad W = gy^T x into the weight's bf16 gradient buffer."""

    @staticmethod
    def forward(ctx, x: Tensor, wb: Tensor, gb: Tensor) -> Tensor:
        x = x.to(wb.dtype)
        ctx.save_for_backward(x)
        ctx.wb, ctx.gb, ctx.side = wb, gb, _SIDE[0]
        return F.linear(x, wb)

    @staticmethod
    def backward(ctx, gy: Tensor):
        (x,) = ctx.saved_tensors
        gy = gy.to(ctx.wb.dtype)
        gb = ctx.gb
        _weight_grad(ctx.side,
                     lambda: torch.mm(gy.reshape(-1, gy.shape[-1]).t(), x.reshape(-1, x.shape[-1]), out=gb),
                     gy, x)
        return gy.matmul(ctx.wb), None, None


class _CachedStacked(torch.autograd.Function):
    """``x3 @ w3b^T`` per slice for a [3, M, C] input and cached [3, N, C] bf16
    weights; the backward writes the three weight gradients into their buffer."""

    @staticmethod
    def forward(ctx, x3: Tensor, w3b: Tensor, g3b: Tensor) -> Tensor:
        x3 = x3.to(w3b.dtype)
        ctx.save_for_backward(x3)
        ctx.w3b, ctx.g3b, ctx.side = w3b, g3b, _SIDE[0]
        return torch.matmul(x3, w3b.transpose(1, 2))

    @staticmethod
    def backward(ctx, gy3: Tensor):
        (x3,) = ctx.saved_tensors
        gy3 = gy3.to(ctx.w3b.dtype)
        g3b = ctx.g3b
        _weight_grad(ctx.side, lambda: torch.bmm(gy3.transpose(1, 2), x3, out=g3b), gy3, x3)
        return torch.matmul(gy3, ctx.w3b), None, None


class _CachedPair(torch.autograd.Function):
    """``x2[0] @ wa^T`` and ``x2[1] @ wb^T`` for a stacked [2, B, T, C] input
    (channel mixing's key and receptance inputs) and cached bf16 weights. The
    backward writes both input gradients into one [2, B, T, C] tensor, the
    stacked gradient the LayerNorm-mix backward reads, where two projections
    of unbound slices would leave autograd to stack them (one copy of both);
    the weight gradients go to their bf16 buffers as in ``_CachedLinear``."""

    @staticmethod
    def forward(ctx, x2: Tensor, wa: Tensor, ga: Tensor, wb: Tensor, gb: Tensor):
        x2 = x2.to(wa.dtype)
        ctx.save_for_backward(x2)
        ctx.ws, ctx.side = ((wa, ga), (wb, gb)), _SIDE[0]
        return F.linear(x2[0], wa), F.linear(x2[1], wb)

    @staticmethod
    def backward(ctx, gya: Tensor, gyb: Tensor):
        (x2,) = ctx.saved_tensors
        c = x2.shape[-1]
        gx2 = torch.empty_like(x2)
        for i, (gy, (w, g)) in enumerate(zip((gya, gyb), ctx.ws)):
            x = x2[i].reshape(-1, c)
            if gy is None:
                gy = x.new_zeros(x.shape[0], w.shape[0])
            gy = gy.to(w.dtype).reshape(-1, w.shape[0])
            _weight_grad(ctx.side, lambda gy=gy, x=x, g=g: torch.mm(gy.t(), x, out=g), gy, x)
            torch.mm(gy, w, out=gx2[i].view(-1, c))
        return gx2, None, None, None, None


class _TimeCore(torch.autograd.Function):
    """``sigmoid(r) * WKV(k, v)`` (the time-mixing core, bf16) from the stacked
    [3, B, T, C] key / value / receptance projections. The same kernels as
    the WKV op and ``fused.gate``, but the backward writes the three
    projection gradients into one [3, B, T, C] tensor, the stacked input of
    the projections' batched weight and input gradients, where separate ops
    on unbound slices would leave autograd to stack them (one copy of all
    three). The saved-state hand-off of the WKV op is kept."""

    @staticmethod
    def forward(ctx, kvr: Tensor, time_decay: Tensor, time_first: Tensor) -> Tensor:
        k, v, rl = kvr.unbind(0)
        state = None
        if _ops.state_saving_enabled():
            y, state = _ops.forward(k, v, time_decay, time_first, save_state=True)
        else:
            y = _ops.forward(k, v, time_decay, time_first)
        ctx.save_for_backward(kvr, time_decay, time_first)
        ctx.y, ctx.state = y, state  # made here, not inputs or outputs
        return fused.gate(rl, y)

    @staticmethod
    def backward(ctx, g: Tensor):
        kvr, time_decay, time_first = ctx.saved_tensors
        y, state = ctx.y, ctx.state
        k, v, rl = kvr.unbind(0)
        gkvr = torch.empty_like(kvr)
        gy = torch.empty_like(y)
        fused.gate_backward_into(g, rl, y, gkvr[2], gy)
        w = -torch.exp(time_decay.float())
        u = time_first.float()
        _gk, _gv, gtd, gtf = _ops.backward(gy, w, u, k, v, state, out=(gkvr[0], gkvr[1]))
        return gkvr, gtd.to(time_decay.dtype), gtf.to(time_first.dtype)


def _linear(x: Tensor, weight: Tensor) -> Tensor:
    """``F.linear(x, weight)``, on the weight's cached bf16 copy when it has one."""
    c = _CACHE.get(id(weight)) if _CACHE else None
    if c is None:
        return F.linear(x, weight)
    return _CachedLinear.apply(x, c[0], c[1])


_BATCHED_KVR = os.environ.get("SPIKEGPT_BATCHED_KVR", "1") != "0"
# With cached weights, the sublayers' projection gradients are produced
# stacked (_TimeCore, _CachedPair); SPIKEGPT_STACKED_GRADS=0: separate ops
# on unbound slices, whose gradients autograd stacks.
_STACKED_GRADS = os.environ.get("SPIKEGPT_STACKED_GRADS", "1") != "0"


class TimeMix(nn.Module):
    """RWKV-4 time mixing (reference SpikeTimeMix, language.py:920-1036)."""

    def __init__(self, n_embd: int, n_layer: int, layer_id: int) -> None:
        super().__init__()
        r01 = layer_id / max(1, n_layer - 1)
        r10 = 1.0 - layer_id / n_layer
        idx = torch.arange(n_embd, dtype=torch.float32)
        self.time_decay = nn.Parameter(-5.0 + 8.0 * torch.pow(idx / max(1, n_embd - 1), 0.7 + 1.3 * r01))
        zigzag = torch.tensor([(i + 1) % 3 - 1 for i in range(n_embd)], dtype=torch.float32)
        self.time_first = nn.Parameter(torch.full((n_embd,), -1.2039728) + 0.5 * zigzag)
        self.time_mix_k = nn.Parameter(_mix_profile(n_embd, r10))
        self.time_mix_v = nn.Parameter(_mix_profile(n_embd, r10, 0.3 * r01))
        self.time_mix_r = nn.Parameter(_mix_profile(n_embd, 0.5 * r10))
        self.key = nn.Linear(n_embd, n_embd, bias=False)
        self.value = nn.Linear(n_embd, n_embd, bias=False)
        self.receptance = nn.Linear(n_embd, n_embd, bias=False)
        self.output = nn.Linear(n_embd, n_embd, bias=False)

    def forward(self, x: Tensor) -> Tensor:
        return self.from_mixed(_shift_mix(x, self.time_mix_k), _shift_mix(x, self.time_mix_v),
                               _shift_mix(x, self.time_mix_r))

    def from_mixed(self, xk: Tensor, xv: Tensor, xr: Tensor) -> Tensor:
        """The sublayer from its three token-shift-mixed inputs."""
        return self._from_projections(_linear(xk, self.key.weight), _linear(xv, self.value.weight),
                                      _linear(xr, self.receptance.weight))

    def from_stacked(self, x3: Tensor) -> Tensor:
        """The sublayer from its three mixed inputs stacked as [3, B, T, C]: the
        key, value and receptance projections (same shape) as one batched GEMM,
        three times the tiles of each alone (the small-batch case fills the GPU)."""
        n, b, t, c = x3.shape
        cached = _CACHE.get((id(self.key.weight), id(self.value.weight), id(self.receptance.weight))) if _CACHE else None
        if cached is not None:
            kvr = _CachedStacked.apply(x3.reshape(n, b * t, c), cached[0], cached[1]).reshape(n, b, t, c)
            if _STACKED_GRADS and fused.gates_supported(kvr[0]):
                return _linear(_TimeCore.apply(kvr, self.time_decay, self.time_first), self.output.weight)
        else:
            w3 = torch.stack([self.key.weight, self.value.weight, self.receptance.weight])
            kvr = torch.matmul(x3.reshape(n, b * t, c), w3.transpose(1, 2)).reshape(n, b, t, c)
        k, v, rl = kvr.unbind(0)
        return self._from_projections(k, v, rl)

    def _from_projections(self, k: Tensor, v: Tensor, rl: Tensor) -> Tensor:
        if k.dtype in (torch.bfloat16, torch.float16):
            wkv = weighted_key_value_cuda_bf16io(k, v, self.time_decay, self.time_first)
        else:
            wkv = weighted_key_value_cuda(k, v, self.time_decay, self.time_first)
        if fused.gates_supported(rl, wkv):  # bf16 autocast: one kernel each way
            return _linear(fused.gate(rl, wkv), self.output.weight)
        return _linear(torch.sigmoid(rl) * wkv, self.output.weight)


class ChannelMix(nn.Module):
    """RWKV-4 channel mixing (reference SpikeChannelMix, language.py:1145-1196)."""

    def __init__(self, n_embd: int, n_layer: int, layer_id: int) -> None:
        super().__init__()
        r10 = 1.0 - layer_id / n_layer
        self.time_mix_k = nn.Parameter(_mix_profile(n_embd, r10))
        self.time_mix_r = nn.Parameter(_mix_profile(n_embd, r10))
        self.key = nn.Linear(n_embd, 4 * n_embd, bias=False)
        self.receptance = nn.Linear(n_embd, n_embd, bias=False)
        self.value = nn.Linear(4 * n_embd, n_embd, bias=False)

    def forward(self, x: Tensor) -> Tensor:
        return self.from_mixed(_shift_mix(x, self.time_mix_k), _shift_mix(x, self.time_mix_r))

    def from_stacked(self, x2: Tensor) -> Tensor:
        """The sublayer from its two mixed inputs stacked as [2, B, T, C]; with
        cached bf16 weights (and bf16 inputs) the two projections are one
        autograd node whose input gradient is that stacked shape."""
        ca = _CACHE.get(id(self.key.weight)) if _CACHE else None
        cb = _CACHE.get(id(self.receptance.weight)) if _CACHE else None
        if not _STACKED_GRADS or ca is None or cb is None or not fused.gates_supported(x2[0]):
            return self.from_mixed(*x2.unbind(0))
        k, r = _CachedPair.apply(x2, ca[0], ca[1], cb[0], cb[1])
        return fused.gate(r, _linear(fused.relu_square(k), self.value.weight))

    def from_mixed(self, xk: Tensor, xr: Tensor) -> Tensor:
        """The sublayer from its two token-shift-mixed inputs. The square is
        taken in the key's dtype: under bf16 autocast, square (pow) would be
        computed in float32 and cast back for the value projection, which
        rounds the same exact square to bf16 once either way. With bf16
        projections the activation and the gate are the fused kernels."""
        k = _linear(xk, self.key.weight)
        if fused.gates_supported(k):  # bf16 autocast: one kernel each way
            v = _linear(fused.relu_square(k), self.value.weight)
            return fused.gate(_linear(xr, self.receptance.weight), v)
        k = torch.relu(k)
        with torch.autocast("cuda", enabled=False):
            k = torch.square(k)
        r = torch.sigmoid(_linear(xr, self.receptance.weight))
        return r * _linear(k, self.value.weight)


class Block(nn.Module):
    """Time mixing and channel mixing, each spiked by a LIF neuron before it
    joins the residual stream (reference SpikeGPTBlock.forward with
    spike_input=False, language.py:1325-1355)."""

    def __init__(self, config: SpikeGPTConfig, layer_id: int) -> None:
        super().__init__()
        c = config.n_embd
        self.config = config
        self.ln0 = nn.LayerNorm(c) if layer_id == 0 else None
        self.ln1 = nn.LayerNorm(c)
        self.ln2 = nn.LayerNorm(c)
        self.att = TimeMix(c, config.n_layer, layer_id)
        self.ffn = ChannelMix(c, config.n_layer, layer_id)
        self.dropout = nn.Dropout(config.dropout)

    def _lif(self, x: Tensor) -> Tensor:
        cfg = self.config
        return surrogate_lif(x, tau=cfg.lif_tau, threshold=cfg.lif_threshold, reset=cfg.lif_reset,
                             surrogate_slope=cfg.surrogate_slope)

    @staticmethod
    def _residual(x: Tensor, spikes: Tensor, token: int = 0) -> Tensor:
        # float32 residual stream + bf16 spikes: one vectorized kernel; with the
        # token of the sublayer's ln_shift_mix, x's gradient is summed in there
        if x.dtype == torch.float32 and spikes.dtype == torch.bfloat16 and x.shape == spikes.shape:
            return fused.residual_add(x, spikes, token)
        return x + spikes

    @staticmethod
    def _fused(x: Tensor) -> bool:
        # Under bf16 autocast the projections take bf16 inputs, which the fused
        # LayerNorm + token-shift kernel produces directly.
        return (torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
                and fused.supported(x))

    def forward(self, x: Tensor, normalized: bool = False) -> Tensor:
        """``normalized``: x already went through this block's ln0."""
        if self.ln0 is not None and not normalized:
            x = self.ln0(x)
        if self._fused(x):
            att, ffn = self.att, self.ffn
            tok = fused.new_residual_token(x)
            x3 = fused.ln_shift_mix_stacked(x, self.ln1.weight, self.ln1.bias,
                                            [att.time_mix_k, att.time_mix_v, att.time_mix_r], self.ln1.eps, tok)
            if _BATCHED_KVR:
                mixed = att.from_stacked(x3)
            else:
                mixed = att.from_mixed(*x3.unbind(0))
            x = self._residual(x, self._lif(mixed), tok)
            tok = fused.new_residual_token(x)
            x2 = fused.ln_shift_mix_stacked(x, self.ln2.weight, self.ln2.bias, [ffn.time_mix_k, ffn.time_mix_r],
                                            self.ln2.eps, tok)
            x = self._residual(x, self._lif(ffn.from_stacked(x2)), tok)
        else:
            x = x + self._lif(self.att(self.ln1(x)))
            x = x + self._lif(self.ffn(self.ln2(x)))
        return self.dropout(x)


class SpikeGPT(nn.Module):
    """Spiking embedding, blocks, final LayerNorm, head; ``forward(ids, targets)``
    returns the mean cross-entropy (reference SpikeLanguageModel.forward /
    loss_tail, language.py:1446-1480)."""

    def __init__(self, config: SpikeGPTConfig = SPIKEGPT_41M) -> None:
        super().__init__()
        config.validate()
        self.config = config
        self.embedding = nn.Embedding(config.vocab_size, config.n_embd)
        self.blocks = nn.ModuleList([Block(config, i) for i in range(config.n_layer)])
        self.ln_out = nn.LayerNorm(config.n_embd)
        self.head = nn.Linear(config.n_embd, config.vocab_size, bias=False)
        for m in self.modules():  # reference _init_weights (language.py:1376-1382)
            if isinstance(m, nn.Embedding):
                nn.init.normal_(m.weight, mean=0.0, std=1.0e-3)
            elif isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, mean=0.0, std=0.01)

    def matmul_weights(self) -> tuple[list[list[nn.Parameter]], nn.Parameter]:
        """The weights of the matrix products: per block, in this order, the
        time mixing's key, value, receptance (the batched projection), output,
        and the channel mixing's key, receptance, value; then the head."""
        groups = [[b.att.key.weight, b.att.value.weight, b.att.receptance.weight, b.att.output.weight,
                   b.ffn.key.weight, b.ffn.receptance.weight, b.ffn.value.weight] for b in self.blocks]
        return groups, self.head.weight

    def forward(self, input_ids: Tensor, targets: Tensor | None = None) -> Tensor:
        if input_ids.ndim != 2:
            raise ValueError(f"input_ids must have shape [B, T]; got {tuple(input_ids.shape)}")
        if input_ids.shape[1] > self.config.context_length:
            raise ValueError("input sequence length exceeds context_length")
        blocks = list(self.blocks)
        ln0 = blocks[0].ln0 if blocks else None
        if ln0 is not None and self.config.vocab_size <= input_ids.numel():
            # The spike and the first block's LayerNorm act row by row, so they
            # commute with the lookup: applied to the table's V rows instead of
            # the batch's B*T tokens (the same forward values; the backward sums
            # the tokens' gradients per row before the LayerNorm's backward
            # instead of after it, which also skips PyTorch's LayerNorm
            # weight-gradient reduction over B*T rows, slow at this shape).
            table = self.embedding.weight
            if self.config.spike_embedding:
                table = _HardSpike.apply(self.config.surrogate_slope * table)
            x = blocks[0](F.embedding(input_ids, ln0(table)), normalized=True)
            blocks = blocks[1:]
        else:
            x = self.embedding(input_ids)
            if self.config.spike_embedding:
                x = _HardSpike.apply(self.config.surrogate_slope * x)
        for block in blocks:
            x = block(x)
        if Block._fused(x):
            # the LayerNorm-mix kernel with a mixing vector of ones is the
            # LayerNorm, rounded to the bf16 the head's product reads (its
            # backward also replaces PyTorch's LayerNorm weight-gradient
            # reduction, slow at this shape)
            ln = self.ln_out
            h = fused.ln_shift_mix_stacked(x, ln.weight, ln.bias, [x.new_ones(x.shape[-1])], ln.eps).squeeze(0)
        else:
            h = self.ln_out(x)
        full, v = _head(h, self.head.weight)
        if targets is None:
            return full[..., :v]
        if full.dtype == torch.bfloat16 and full.is_cuda:  # bf16 autocast: the fused loss, logits read in place
            return fused.cross_entropy(full.reshape(-1, full.shape[-1]), targets, v)
        logits = full[..., :v]
        return F.cross_entropy(logits.reshape(-1, v).float(), targets.reshape(-1))


def _head(h: Tensor, weight: Tensor, multiple: int = 64) -> tuple[Tensor, int]:
    """The output projection ``h @ weight.T``: (logits [.., Vp], V), the first V
    columns the classes. When V is not a multiple of 64 (the GPT-2 BPE
    vocabulary, 50257) on CUDA, the weight is zero-padded to Vp, a multiple of
    64, for the product: with an odd V the library GEMM falls back to an
    alignment-1 kernel at a few percent of the tensor peak (54 of 115 ms of the
    216M-class step). The padded columns are never read as classes, so values
    and gradients are those of the plain projection."""
    v = weight.shape[0]
    c = _CACHE.get(id(weight)) if _CACHE else None
    if c is not None:  # the cached copy is stored padded (zero rows past V)
        return _CachedLinear.apply(h, c[0], c[1]), v
    pad = (-v) % multiple
    if pad == 0 or not h.is_cuda:
        return F.linear(h, weight), v
    return F.linear(h, F.pad(weight, (0, 0, 0, pad))), v


def head_rows(v: int, multiple: int = 64) -> int:
    """Rows of the head weight as ``_head`` multiplies by it on CUDA."""
    return v + (-v) % multiple


def parameter_count(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())


def flops_per_token(config: SpikeGPTConfig) -> float:
    """Model FLOPs per token for MFU: 6 x the weights of the matrix products
    (forward and backward), 13 C^2 per layer (time mixing 4 C^2, channel
    mixing 9 C^2) plus the head C x V; the embedding lookup, WKV, LIF and
    elementwise terms are left out. 246.2 MFLOP for SpikeGPT-41M."""
    c, v = config.n_embd, config.vocab_size
    return 6.0 * (config.n_layer * 13 * c * c + c * v)
