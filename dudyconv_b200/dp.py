"""Data-parallel helpers for the fused dynamic conv.

The op shards over independent sequences: every rank runs its own slice of the batch,
``kernel_mix`` is replicated, and the only exchange is the sum of ``grad_kernel_mix`` over
ranks after the backward. The sum is taken in fp32 (the per-rank values are fp32 sums cast
to the input dtype) and cast back, so the reduction itself adds no 16-bit rounding.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(batch: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of the sequences owned by `rank` (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world: {rank}/{world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def allreduce_grad_mix(grad_mix: torch.Tensor, group=None, async_op: bool = False):
    """Sum `grad_mix` over the process group in place (fp32 accumulation).

    Returns the async work handle when `async_op` is true (the caller waits on it before
    reading `grad_mix`), else None.
    """
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return None
    if grad_mix.dtype == torch.float32:
        return dist.all_reduce(grad_mix, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
    buf = grad_mix.float()
    work = dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
    if async_op:
        class _Work:
            def wait(self_inner):
                work.wait()
                grad_mix.copy_(buf)
        return _Work()
    grad_mix.copy_(buf)
    return None
