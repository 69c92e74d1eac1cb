"""Data-parallel train step of the SpikeGPT model with the forward and backward
replayed from one CUDA graph.

The reference trains with eager PyTorch under DDP (src/spikegpt/train.py and
its model, language.py:1361-1480). An eager step of SpikeGPT-41M launches
about 1100 kernels; at 64 sequences per GPU their device time dominates, but
with the batch split over 2 to 8 GPUs each kernel shrinks while the host time
to launch it does not, and the step turns launch-bound. Here the forward and
backward are captured once and replayed, so the host issues one graph launch,
one all-reduce and the fused optimizer per step.

Gradients: the backward starts from ``.grad = None``, so autograd hands each
parameter the gradient tensor it produced (no zero fill, no accumulation
kernels). On one rank the optimizer reads those. On several, one
concatenation (captured with the backward) gathers them into a flat float32
buffer (in backward order), a single all-reduce averages it (DDP's average of
the ranks' gradients of their shard-mean losses: ``ReduceOp.AVG`` over NCCL;
gloo sums and divides), and the parameters' ``.grad`` are views of that buffer
for the optimizer. The all-reduce and the optimizer step run outside the
graph, on the current stream.

``overlap=True`` instead all-reduces the gradients in buckets of about 25 MB
while the backward runs (DDP's bucketing): a hook on each parameter counts the
gradients of its bucket, and the bucket's last gradient gathers them into its
slice of the flat buffer and starts an asynchronous all-reduce; with a CUDA
graph the all-reduces are captured with the backward. On two B200s over NVLink
it measured slower than the single all-reduce afterwards (SpikeGPT-41M, 32
sequences per GPU: 21.07 against 20.64 ms per step; 8 per GPU: 8.57 against
8.51 ms; the all-reduce of 165 MB takes 0.41 ms), so it is off by default.

``graph=False`` runs the same step eagerly (any device, any process group:
the CPU tests use it over gloo).

Weight cache (bf16 autocast on CUDA, a model with ``matmul_weights()``, no
bucketed overlap): the matmul weights live in one flat float32 buffer (the
parameters become views of it); each step casts it to a flat bf16 copy with
one kernel, the projections multiply by the copies (``model.weight_cache``)
and write their bf16 weight gradients into a flat bf16 buffer, which one more
kernel widens into the flat float32 gradient buffer: [matmul weights | head |
the other parameters in backward order], of which every parameter's ``.grad``
is a view. This replaces autocast's per-weight casts (about 200 kernels a step
in SpikeGPT-41M) with four, and computes the same values. The weight-gradient
products run on a side stream (``side_wgrad``), joined before the widening:
they overlap the rest of the backward.
"""

from __future__ import annotations

import contextlib

import torch
import torch.distributed as dist
from torch import Tensor, nn

from . import _capi, fused


class TrainStep:
    """One optimizer step of ``model(ids, targets) -> loss`` per call.

    ``batch_shape`` is the (rows, T) shape of this rank's token ids and
    targets; every call must pass that shape. ``group`` is the data-parallel
    process group (None: the default group when one is initialized, else no
    exchange). ``autocast_dtype`` None runs without autocast.
    """

    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer, batch_shape: tuple[int, int], *,
                 device: torch.device | str, autocast_dtype: torch.dtype | None = torch.bfloat16,
                 graph: bool = True, group=None, warmup: int = 3, overlap: bool = False,
                 bucket_mb: float = 25.0, weight_cache: bool = True, side_wgrad: bool = True,
                 micro_batches: int = 1) -> None:
        self.model = model
        self.optimizer = optimizer
        self.device = torch.device(device)
        self.autocast_dtype = autocast_dtype
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        # NCCL averages in the collective; gloo has no AVG, so it sums and divides
        self.avg = self.world > 1 and dist.get_backend(group) == "nccl"
        if graph and self.device.type != "cuda":
            raise ValueError("graph capture needs a CUDA device")
        params = [p for p in model.parameters() if p.requires_grad]
        if any(p.device != self.device or p.dtype != torch.float32 for p in params):
            raise ValueError("TrainStep expects float32 parameters on its device")
        self.params = params
        self.grads = None  # the flat gradient buffer (several ranks only)
        self.grad_views = None
        self.overlap = overlap and self.world > 1
        self.buckets: list[tuple[list[nn.Parameter], Tensor]] = []
        self.cache = None  # weight cache entries (see the module docstring)
        self.cached_ids: set[int] = set()
        self.side = None  # the stream of the cached projections' weight gradients
        self.micro = int(micro_batches)
        if self.micro < 1 or batch_shape[0] % self.micro:
            raise ValueError(f"micro_batches={micro_batches} must divide the {batch_shape[0]} rows")
        if (weight_cache and autocast_dtype == torch.bfloat16 and self.device.type == "cuda"
                and not self.overlap and hasattr(model, "matmul_weights")):
            self._build_cache()
            if side_wgrad:
                self.side = torch.cuda.Stream(self.device)
            self.mb_streams = [torch.cuda.Stream(self.device) for _ in range(self.micro)] if self.micro > 1 else []
        elif self.micro > 1:
            raise ValueError("micro_batches > 1 needs the weight cache (bf16 autocast on CUDA, no overlap)")
        elif self.world > 1:
            self._layout(bucket_mb)
        self.ids = torch.zeros(batch_shape, dtype=torch.long, device=self.device)
        self.targets = torch.zeros(batch_shape, dtype=torch.long, device=self.device)
        self.graph = None
        self.loss = None
        self.captured_grads = None
        self.captured_launches = 0  # this package's kernels in the graph (each replay runs them again)
        self._ar_events: list[tuple[torch.cuda.Event, torch.cuda.Event]] | None = None
        if graph:
            self._capture(warmup)

    def _layout(self, bucket_mb: float) -> None:
        """Flat gradient buffer in backward order (the reverse of registration,
        which follows the forward), cut into buckets of about bucket_mb MB."""
        order = list(reversed(self.params))
        self.grads = torch.zeros(sum(p.numel() for p in order), dtype=torch.float32, device=self.device)
        limit = max(1, int(bucket_mb * 2**20 / 4))
        view_of: dict[int, Tensor] = {}
        off, start, members = 0, 0, []
        for p in order:
            view_of[id(p)] = self.grads[off:off + p.numel()].view_as(p)
            members.append(p)
            off += p.numel()
            if off - start >= limit or p is order[-1]:
                self.buckets.append((members, self.grads[start:off]))
                start, members = off, []
        self.grad_views = [view_of[id(p)] for p in self.params]
        self._bucket_of = {id(p): i for i, (ms, _) in enumerate(self.buckets) for p in ms}
        self._ready = [0] * len(self.buckets)
        self._works: list = []
        self._collecting = False
        if self.overlap:
            for p in self.params:
                p.register_post_accumulate_grad_hook(self._grad_ready)

    def _build_cache(self) -> None:
        from .model import head_rows

        groups, head = self.model.matmul_weights()
        mm = [p for g in groups for p in g]
        ids = {id(p) for p in mm} | {id(head)}
        owned = {id(p) for p in self.params}
        if len(ids) != len(mm) + 1 or not ids <= owned:
            raise ValueError("matmul_weights() must list distinct trainable parameters")
        dev = self.device
        n = sum(p.numel() for p in mm)
        v, c = head.shape
        self.w32 = torch.empty(n, dtype=torch.float32, device=dev)
        self.w16 = torch.empty(n, dtype=torch.bfloat16, device=dev)
        # the head's copy is stored with the zero rows _head pads to
        self.h16 = torch.zeros(head_rows(v), c, dtype=torch.bfloat16, device=dev)
        # bf16 weight-gradient buffers, one set per micro-batch
        self.g16s = [torch.empty(n, dtype=torch.bfloat16, device=dev) for _ in range(self.micro)]
        self.hg16s = [torch.zeros(head_rows(v), c, dtype=torch.bfloat16, device=dev) for _ in range(self.micro)]
        self.caches = [{} for _ in range(self.micro)]
        off = 0
        for g in groups:
            start = off
            for p in g:
                k = p.numel()
                self.w32[off:off + k].copy_(p.detach().reshape(-1))
                p.data = self.w32[off:off + k].view_as(p)
                for e, g16 in zip(self.caches, self.g16s):
                    e[id(p)] = (self.w16[off:off + k].view_as(p), g16[off:off + k].view_as(p))
                off += k
            kk, vv, rr = g[0], g[1], g[2]  # the batched key / value / receptance projection
            if kk.shape == vv.shape == rr.shape:
                m = 3 * kk.numel()
                for e, g16 in zip(self.caches, self.g16s):
                    e[(id(kk), id(vv), id(rr))] = (self.w16[start:start + m].view(3, *kk.shape),
                                                   g16[start:start + m].view(3, *kk.shape))
        for e, hg16 in zip(self.caches, self.hg16s):
            e[id(head)] = (self.h16, hg16)
        self.head = head
        self.cache = self.caches[0]
        self.cached_ids = ids
        self.others = [p for p in reversed(self.params) if id(p) not in ids]
        self.n_mm, self.n_head_end = n, n + head.numel()
        self.grads = torch.zeros(self.n_head_end + sum(p.numel() for p in self.others),
                                 dtype=torch.float32, device=dev)
        view_of: dict[int, Tensor] = {}
        off = 0
        for p in mm + [head] + self.others:
            view_of[id(p)] = self.grads[off:off + p.numel()].view_as(p)
            off += p.numel()
        self.grad_views = [view_of[id(p)] for p in self.params]
        for p in mm + [head]:
            p.grad = view_of[id(p)]

    def _grad_ready(self, p: Tensor) -> None:
        # autograd hook: p.grad is final for this backward
        if not self._collecting:
            return
        i = self._bucket_of[id(p)]
        self._ready[i] += 1
        if self._ready[i] == len(self.buckets[i][0]):
            self._reduce_bucket(i)

    def _reduce_bucket(self, i: int) -> None:
        members, flat = self.buckets[i]
        grads = [p.grad.reshape(-1) if p.grad is not None else torch.zeros(p.numel(), device=self.device)
                 for p in members]
        torch.cat(grads, out=flat)
        op = dist.ReduceOp.AVG if self.avg else dist.ReduceOp.SUM
        self._works.append((i, dist.all_reduce(flat, op=op, group=self.group, async_op=True)))
        self._ready[i] = -1  # launched

    def _finish_buckets(self) -> None:
        """Launch the buckets the hooks did not (parameters without a gradient)
        and make the current stream wait for every bucket's all-reduce."""
        for i, n in enumerate(self._ready):
            if n != -1:
                self._reduce_bucket(i)
        for i, work in self._works:
            work.wait()
            if not self.avg:
                self.buckets[i][1].div_(self.world)
        self._works = []
        self._ready = [0] * len(self.buckets)

    def _forward_backward(self) -> Tensor:
        from .model import side_operands, weight_cache

        for p in self.params:
            if id(p) not in self.cached_ids:
                p.grad = None
        cache = contextlib.nullcontext()
        if self.cache is not None:  # this step's bf16 copies of the matmul weights
            self.w16.copy_(self.w32)
            self.h16[:self.head.shape[0]].copy_(self.head.detach())
            cache = weight_cache(self.cache, self.side)
        # the full backward below consumes every skip gradient handed over
        # between a residual_add and its LayerNorm-mix (fused.residual_handoff)
        self._collecting = self.overlap
        try:
            if self.micro > 1:
                loss = self._micro_forward_backward()
            else:
                with fused.residual_handoff(), cache:
                    if self.autocast_dtype is None:
                        loss = self.model(self.ids, self.targets)
                    else:
                        with torch.autocast(self.device.type, dtype=self.autocast_dtype):
                            loss = self.model(self.ids, self.targets)
                    loss.backward()
        finally:
            self._collecting = False
        if fused.pending_residual_grads():
            fused.drop_residual_grads()
            raise RuntimeError("TrainStep: a residual gradient was handed over but never consumed")
        fused.drop_residual_grads()  # bf16 grad-x copies no residual_add took (the first sublayer's)
        if self.cache is not None:
            if self.side is not None:  # the weight gradients written on the side stream
                torch.cuda.current_stream(self.device).wait_stream(self.side)
                side_operands().clear()
            gmm, ghead = self.grads[:self.n_mm], self.grads[self.n_mm:self.n_head_end].view_as(self.head)
            v = self.head.shape[0]
            gmm.copy_(self.g16s[0])
            ghead.copy_(self.hg16s[0][:v])
            for g16, hg16 in zip(self.g16s[1:], self.hg16s[1:]):  # the other micro-batches' shares
                gmm.add_(g16)
                ghead.add_(hg16[:v])
            torch.cat([p.grad.reshape(-1) for p in self.others], out=self.grads[self.n_head_end:])
        elif self.overlap:
            self._finish_buckets()
        elif self.grads is not None:
            torch.cat([p.grad.reshape(-1) for p in reversed(self.params)], out=self.grads)
        return loss.detach()

    def _micro_forward_backward(self) -> Tensor:
        """Forward and backward of the rank's batch as ``micro`` micro-batches,
        each on its own stream: autograd runs each backward op on the stream of
        its forward op, so the micro-batches' kernels overlap (at a few
        sequences per GPU most kernels leave SMs idle). Each micro-batch writes
        its own bf16 weight gradients; the loss is the mean of the micro-batch
        means (equal sizes: the batch mean)."""
        from .model import weight_cache

        cur = torch.cuda.current_stream(self.device)
        rows = self.ids.shape[0] // self.micro
        losses = []
        with fused.residual_handoff():
            for i, s in enumerate(self.mb_streams):
                s.wait_stream(cur)
                sl = slice(i * rows, (i + 1) * rows)
                with torch.cuda.stream(s), weight_cache(self.caches[i], self.side), \
                        torch.autocast(self.device.type, dtype=self.autocast_dtype):
                    losses.append(self.model(self.ids[sl], self.targets[sl]))
            for s in self.mb_streams:
                cur.wait_stream(s)
            loss = torch.stack(losses).mean()
            loss.backward()
        for s in self.mb_streams:
            cur.wait_stream(s)
        return loss

    def _capture(self, warmup: int) -> None:
        # Warm-up on a side stream (as graph capture requires), then capture.
        # Neither touches the parameters: the optimizer does not run here.
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                self._forward_backward()
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        before = sum(_capi.launch_counts().values())
        with torch.cuda.graph(self.graph):
            self.loss = self._forward_backward()
        self.captured_launches = sum(_capi.launch_counts().values()) - before
        # every replay rewrites the gradient tensors the capture produced
        self.captured_grads = [p.grad for p in self.params]
        if self.grad_views is not None:
            for p, g in zip(self.params, self.grad_views):
                p.grad = g

    def __call__(self, ids: Tensor, targets: Tensor) -> Tensor:
        """Copy the batch in, run forward and backward, average the gradients
        over the ranks, step the optimizer. Returns the loss of this rank's
        shard (a device tensor; with a graph, the same tensor every call)."""
        if tuple(ids.shape) != tuple(self.ids.shape) or tuple(targets.shape) != tuple(self.targets.shape):
            raise ValueError(f"batch shape {tuple(ids.shape)} differs from the captured {tuple(self.ids.shape)}")
        self.ids.copy_(ids, non_blocking=True)
        self.targets.copy_(targets, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
            loss = self.loss
        else:
            loss = self._forward_backward()
        if self.grads is not None and self.world > 1 and not self.overlap:
            ev = None
            if self._ar_events is not None:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
            if self.avg:
                dist.all_reduce(self.grads, op=dist.ReduceOp.AVG, group=self.group)
            else:
                dist.all_reduce(self.grads, op=dist.ReduceOp.SUM, group=self.group)
                self.grads.div_(self.world)
            if ev is not None:
                ev[1].record()
                self._ar_events.append(ev)
        if self.grads is not None:
            if self.graph is None:
                for p, g in zip(self.params, self.grad_views):
                    p.grad = g
        self.optimizer.step()
        return loss

    def time_allreduce(self, on: bool = True) -> None:
        """Record CUDA events around each call's gradient all-reduce (on the
        current stream) until ``allreduce_ms`` collects them; only the
        all-reduce after the backward (overlap=False) is timed."""
        self._ar_events = [] if on else None

    def allreduce_ms(self) -> tuple[float, int]:
        """(summed device ms, count) of the all-reduces timed since
        ``time_allreduce(True)``; synchronizes on the last one."""
        evs = self._ar_events or []
        if evs:
            evs[-1][1].synchronize()
        total = sum(a.elapsed_time(b) for a, b in evs)
        if self._ar_events is not None:
            self._ar_events = []
        return total, len(evs)

    def release(self) -> None:
        """Drop the captured graph (before the process group is destroyed)."""
        self.graph = None
        self.loss = None
        self.captured_grads = None
