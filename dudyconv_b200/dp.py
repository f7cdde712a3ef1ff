"""Data-parallel helpers for the fused dynamic conv.

The op shards over independent sequences: every rank runs its own slice of the batch,
``kernel_mix`` is replicated, and the only exchange is the sum of ``grad_kernel_mix`` over
ranks after the backward. For sequences too long for one GPU it also shards along time
(``sequence_sharded_dynamic_conv``) with one causal halo exchange between neighbours. The sum is taken in fp32 (the per-rank values are fp32 sums cast
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


class GradMixExchange:
    """Peer-memory buffers for the data-parallel backward (``dudy_fdc_backward_dp``).

    Each rank allocates one exchange buffer of ``dudy_fdc_exchange_bytes(D, N)`` bytes as
    symmetric memory (``torch.distributed._symmetric_memory``: the same allocation mapped
    in every rank's process over NVLink), zero-fills it, and learns every peer's address.
    ``backward`` then runs this rank's backward and sums grad_mix over the ranks in the
    backward's last kernel, over peer memory, instead of a separate all-reduce. Every rank
    must call ``backward`` the same number of times (the call counter is the exchange's
    epoch), one rank per GPU.
    """

    def __init__(self, D: int, N: int, group=None, device=None):
        import torch.distributed._symmetric_memory as symm_mem

        from . import capi

        self.capi = capi
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        if self.world > capi.MAX_PEERS:
            raise ValueError(f"at most {capi.MAX_PEERS} ranks, got {self.world}")
        nbytes = capi.fdc_exchange_bytes(D, N)
        dev = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.buf = symm_mem.empty((nbytes + 15) // 16 * 4, dtype=torch.float32, device=dev)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, self.group.group_name)
        base = self.handle.buffer_ptrs[self.rank]
        offset = self.buf.data_ptr() - base
        self.desc = capi.PeerExchange()
        for r, p in enumerate(self.handle.buffer_ptrs):
            self.desc.bufs[r] = p + offset
        self.desc.rank, self.desc.world, self.desc.epoch = self.rank, self.world, 0
        # every rank's buffer must be zero before any rank publishes into it
        torch.cuda.synchronize(dev)
        dist.barrier(self.group)

    def backward(self, go, h, kc, mix, grad_h, grad_kc, grad_mix, workspace, off: int,
                 dilation: int, plan: int = -1, stream=None):
        """Synchronous: grad_mix gets this call's sum over ranks."""
        self.desc.epoch += 1
        self.capi.fdc_backward_dp(go, h, kc, mix, grad_h, grad_kc, grad_mix, workspace,
                                  self.desc, off, dilation, plan, stream)

    def backward_deferred(self, go, h, kc, mix, grad_h, grad_kc, grad_mix, grad_mix_prev,
                          workspace, off: int, dilation: int, plan: int = -1, stream=None):
        """Deferred: grad_mix gets this rank's own sum, grad_mix_prev the sum over ranks of
        the previous call (untouched on the first call); ``finish`` gives the last one."""
        self.desc.epoch += 1
        self.capi.fdc_backward_dp_deferred(go, h, kc, mix, grad_h, grad_kc, grad_mix,
                                           grad_mix_prev, workspace, self.desc, off, dilation,
                                           plan, stream)

    def finish(self, grad_mix, stream=None):
        """The sum over ranks of the last call into grad_mix."""
        self.capi.fdc_exchange_finish(self.desc, grad_mix, stream)


# ---------------------------------------------------------------------------------------
# Sequence sharding: one causal halo exchange per call
# ---------------------------------------------------------------------------------------
def _neighbours(group):
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    prev = dist.get_global_rank(group, rank - 1) if group is not None and rank > 0 else rank - 1
    nxt = dist.get_global_rank(group, rank + 1) if group is not None and rank + 1 < world else rank + 1
    return rank, world, prev, nxt


def _exchange(send_to, send_t, recv_from, recv_t, group):
    """Send `send_t` to rank `send_to` and receive `recv_t` from `recv_from` (either may be
    None); both transfers are posted before either is waited on."""
    ops = []
    if send_to is not None:
        ops.append(dist.P2POp(dist.isend, send_t, send_to, group))
    if recv_from is not None:
        ops.append(dist.P2POp(dist.irecv, recv_t, recv_from, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


class HaloExchange(torch.autograd.Function):
    """Forward: rank r receives the last `halo` positions of rank r-1's `h_local` (zeros on
    rank 0) and sends its own last `halo` positions to rank r+1. Backward: the gradient of the
    received halo goes back to rank r-1 and is added to its last `halo` positions."""

    @staticmethod
    def forward(ctx, h_local, halo, group):
        rank, world, prev, nxt = _neighbours(group)
        ctx.halo, ctx.group = halo, group
        recv = torch.zeros(*h_local.shape[:-1], halo, dtype=h_local.dtype, device=h_local.device)
        send = h_local[..., h_local.shape[-1] - halo:].contiguous()
        _exchange(nxt if rank + 1 < world else None, send, prev if rank > 0 else None, recv, group)
        ctx.local_len = h_local.shape[-1]
        return recv

    @staticmethod
    def backward(ctx, grad_recv):
        rank, world, prev, nxt = _neighbours(ctx.group)
        halo = ctx.halo
        back = torch.zeros(*grad_recv.shape, dtype=grad_recv.dtype, device=grad_recv.device)
        _exchange(prev if rank > 0 else None, grad_recv.contiguous(),
                  nxt if rank + 1 < world else None, back, ctx.group)
        grad = torch.zeros(*grad_recv.shape[:-1], ctx.local_len, dtype=grad_recv.dtype,
                           device=grad_recv.device)
        grad[..., ctx.local_len - halo:] = back
        return grad, None, None


def sequence_sharded_dynamic_conv(h_local, kernel_local, kernel_mix, dilation: int = 1,
                                  group=None, op=None):
    """fused_dynamic_conv over a sequence split along time across the ranks of `group`.

    Rank r holds positions [r*Ls, (r+1)*Ls) of every sequence: `h_local` [B,D,Ls] and
    `kernel_local` [B,K,N,Ls]; `kernel_mix` [D,N] is replicated. The causal window reaches
    H = (K-1)*dilation positions back, so each rank takes those H positions from its
    predecessor (one exchange with each neighbour per forward and per backward) and runs the
    op on [halo | h_local] with t_offset = H. Returns this rank's output [B,D,Ls]. Gradients
    reach `h_local` (including the halo positions the successor used), `kernel_local` and
    `kernel_mix`; sum `kernel_mix.grad` over the group afterwards (allreduce_grad_mix).
    Requires H <= Ls (the halo comes from one neighbour).

    `op(h_full, kernel_chunk, kernel_mix, t_offset, dilation)` defaults to
    dudyconv_b200.cuda_ops.fused_dynamic_conv_chunk.
    """
    if op is None:
        from .cuda_ops import fused_dynamic_conv_chunk as op
    K = kernel_local.shape[1]
    halo = (K - 1) * int(dilation)
    Ls = h_local.shape[-1]
    if kernel_local.shape[-1] != Ls:
        raise ValueError("kernel_local must cover the same positions as h_local")
    if halo > Ls:
        raise ValueError(f"causal span {halo} exceeds the local length {Ls}")
    if halo == 0 or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return op(h_local, kernel_local, kernel_mix, 0, int(dilation))
    recv = HaloExchange.apply(h_local, halo, group)
    h_ext = torch.cat([recv, h_local], dim=-1)
    return op(h_ext, kernel_local, kernel_mix, halo, int(dilation))
