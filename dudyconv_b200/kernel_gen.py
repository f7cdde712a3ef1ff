"""The kernel generator's tail as one fused pass, and the op taking logits directly.

In the reference model the dynamic conv's ``kernel_chunk`` comes out of
``StreamingKernelGenConv1d._logits_to_kernel`` (``backbone_dil_unshared.py:1821-1900``):
the generator's logits ``[B, N*K, T]`` are viewed as ``[B, N, K, T]``, soft-maxed over K,
flipped along K (so that tap ``kk = 0`` is the current token) and permuted into the
contiguous ``[B, K, N, T]`` layout the op reads. PyTorch runs that as three full passes
over the tensor forward (softmax, flip copy, permute copy) and three backward.

``logits_to_kernel`` does it in one pass each way (``dudy_logits_to_kernel`` /
``dudy_logits_to_kernel_backward`` in the C ABI): read the logits once and write
``kernel_chunk`` once; backward, read ``kernel_chunk`` and its gradient once and write the
logits' gradient once. ``fused_dynamic_conv_chunk_from_logits`` is the op fed straight
from the logits (the op's backward needs ``kernel_chunk`` itself, so it is written once
and kept, as autograd keeps it in the reference).

Nothing here replaces the reference's API; these are additions beside it.
"""

from __future__ import annotations

import torch

from . import load_extension
from .cuda_ops.fused_dynamic_conv import fused_dynamic_conv_chunk

_EXT = load_extension()


class LogitsToKernelFunction(torch.autograd.Function):
    """logits [B, N*K, T] -> kernel_chunk [B, K, N, T]: softmax over K, then flip K."""

    @staticmethod
    def forward(ctx, logits, num_kernels: int, kernel_size: int):
        if not logits.is_cuda:
            raise RuntimeError("logits must be CUDA tensor.")
        kc = _EXT.logits_to_kernel(logits.contiguous(), int(num_kernels), int(kernel_size))
        ctx.save_for_backward(kc)
        return kc

    @staticmethod
    def backward(ctx, grad_kc):
        (kc,) = ctx.saved_tensors
        grad_logits = _EXT.logits_to_kernel_backward(kc, grad_kc.contiguous())
        return grad_logits, None, None


def logits_to_kernel(logits: torch.Tensor, num_kernels: int, kernel_size: int) -> torch.Tensor:
    """Fused ``_logits_to_kernel``: ``[B, N*K, T]`` logits -> ``[B, K, N, T]`` kernel."""
    return LogitsToKernelFunction.apply(logits, num_kernels, kernel_size)


def fused_dynamic_conv_chunk_from_logits(h_full: torch.Tensor, kernel_logits: torch.Tensor,
                                         kernel_mix: torch.Tensor, t_offset: int = 0,
                                         dilation: int = 1) -> torch.Tensor:
    """``fused_dynamic_conv_chunk(h_full, _logits_to_kernel(kernel_logits), kernel_mix, ...)``
    with the logits-to-kernel step fused: ``kernel_logits`` is the kernel generator's
    ``[B, N*K, T]`` output, N taken from ``kernel_mix`` ``[D, N]``."""
    if kernel_logits.dim() != 3:
        raise RuntimeError(f"kernel_logits must be [B,N*K,T], got {tuple(kernel_logits.shape)}.")
    N = int(kernel_mix.shape[1])
    if kernel_logits.shape[1] % N != 0:
        raise RuntimeError(f"kernel_logits channels ({kernel_logits.shape[1]}) are not a "
                           f"multiple of N={N}.")
    kc = logits_to_kernel(kernel_logits, N, kernel_logits.shape[1] // N)
    return fused_dynamic_conv_chunk(h_full, kc, kernel_mix, t_offset, dilation)
