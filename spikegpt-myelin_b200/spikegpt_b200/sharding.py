"""Batch sharding of the WKV op across ranks (one process per GPU).

Every (batch, channel) lane of the recurrence is independent, so a data-parallel
job gives each rank a contiguous slice of the batch and runs the op on it with
no communication in the forward or backward. The only exchange is the one a
data-parallel step already does for its parameters: the per-channel gradients
``grad_time_decay`` and ``grad_time_first`` (sums over the batch,
reference src/spikegpt/wkv_triton.py:194) are summed over ranks, after which
every rank holds the full-batch values.

The helpers take any ``torch.distributed`` process group: NCCL on GPUs, gloo
for the CPU tests.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [start, stop) of a batch of ``batch`` rows owned by ``rank``.

    Contiguous, in rank order, sizes differing by at most one (the first
    ``batch % world`` ranks get the extra row); a rank may get zero rows.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if batch < 0:
        raise ValueError(f"batch must be >= 0, got {batch}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def reduce_channel_grads(*grads: torch.Tensor, group=None) -> None:
    """Sum per-channel gradients ([C] tensors) over ranks, in place.

    One flattened all-reduce for all of them, so ranks issue exactly one
    collective per call whatever the number of tensors.
    """
    if not grads:
        return
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    flat = torch.cat([g.reshape(-1).to(torch.float32) for g in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n


def max_over_ranks(value: float, device: torch.device | str = "cpu", group=None) -> float:
    """The maximum of a per-rank number (a device time in ms) over all ranks."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
