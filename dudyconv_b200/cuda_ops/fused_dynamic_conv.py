"""Fused dynamic causal convolution: the public Python API.

Same names, signatures, argument meaning, defaults and error messages as the
reference's ``cuda_ops/fused_dynamic_conv.py`` (adjfangjiawei/DUDyConv), so callers
(``backbone_dil_unshared.py``, the reference tests) run unchanged. The compute goes to
the in-tree ``cuda_ops_ext`` binding (tcgen05/TMEM kernels for fp16/bf16 hot shapes,
CUDA-core kernels otherwise); there is no CPU path.

Layout (reference ``cuda_ops/fused_dynamic_conv.py:7-31``)::

    h_full       [B, D, L]   contiguous CUDA, fp32 / fp16 / bf16
    kernel_chunk [B, K, N, T] same dtype
    kernel_mix   [D, N]       same dtype
    out          [B, D, T]
    out[b,d,t] = sum_kk sum_n h_full[b,d,t_offset+t-kk*dilation]
                              * kernel_chunk[b,kk,n,t] * kernel_mix[d,n]
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import load_extension

_EXT = load_extension()

_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


# ---------------------------------------------------------------------------------------
# input checks (reference cuda_ops/fused_dynamic_conv.py:108-235)
# ---------------------------------------------------------------------------------------
def _check_forward_inputs(h_full, kernel_chunk, kernel_mix, t_offset, dilation) -> None:
    t_offset, dilation = int(t_offset), int(dilation)
    if dilation <= 0:
        raise RuntimeError("dilation must be positive.")
    for name, t in (("h_full", h_full), ("kernel_chunk", kernel_chunk), ("kernel_mix", kernel_mix)):
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be CUDA tensor.")
    if h_full.dim() != 3:
        raise RuntimeError(f"h_full must be [B,D,L], got {tuple(h_full.shape)}.")
    if kernel_chunk.dim() != 4:
        raise RuntimeError(f"kernel_chunk must be [B,K,N,T], got {tuple(kernel_chunk.shape)}.")
    if kernel_mix.dim() != 2:
        raise RuntimeError(f"kernel_mix must be [D,N], got {tuple(kernel_mix.shape)}.")
    B, D, L = h_full.shape
    Bk, K, N, T = kernel_chunk.shape
    Dm, Nm = kernel_mix.shape
    if B != Bk:
        raise RuntimeError(f"B mismatch: h_full={B}, kernel_chunk={Bk}.")
    if D != Dm:
        raise RuntimeError(f"D mismatch: h_full={D}, kernel_mix={Dm}.")
    if N != Nm:
        raise RuntimeError(f"N mismatch: kernel_chunk={N}, kernel_mix={Nm}.")
    if T <= 0:
        raise RuntimeError("T must be positive.")
    if K <= 0:
        raise RuntimeError("K must be positive.")
    if t_offset < 0:
        raise RuntimeError("t_offset must be non-negative.")
    if t_offset + T > L:
        raise RuntimeError(
            f"t_offset + T must be <= L, got t_offset={t_offset}, T={T}, L={L}.")
    if h_full.dtype not in _DTYPES:
        raise RuntimeError(f"Unsupported dtype: {h_full.dtype}.")
    if kernel_chunk.dtype != h_full.dtype:
        raise RuntimeError("kernel_chunk dtype must equal h_full dtype.")
    if kernel_mix.dtype != h_full.dtype:
        raise RuntimeError("kernel_mix dtype must equal h_full dtype.")


def _check_backward_inputs(grad_out, h_full, kernel_chunk, kernel_mix, t_offset, dilation) -> None:
    _check_forward_inputs(h_full, kernel_chunk, kernel_mix, t_offset, dilation)
    if not grad_out.is_cuda:
        raise RuntimeError("grad_out must be CUDA tensor.")
    if grad_out.dim() != 3:
        raise RuntimeError(f"grad_out must be [B,D,T], got {tuple(grad_out.shape)}.")
    B, D, _ = h_full.shape
    T = kernel_chunk.shape[3]
    for axis, (want, label) in enumerate(((B, "h_full"), (D, "h_full"), (T, "kernel_chunk T"))):
        if grad_out.shape[axis] != want:
            dim = "BDT"[axis]
            raise RuntimeError(
                f"grad_out {dim} mismatch: grad_out={grad_out.shape[axis]}, {label}={want}.")
    if grad_out.dtype != h_full.dtype:
        raise RuntimeError("grad_out dtype must equal h_full dtype.")


def _check_backward_plan_inputs(h_full, kernel_chunk, t_offset, dilation) -> None:
    """Checks of the cached-backward-plan query (reference :444-523): no kernel_mix."""
    t_offset, dilation = int(t_offset), int(dilation)
    if dilation <= 0:
        raise RuntimeError("dilation must be positive.")
    if not h_full.is_cuda:
        raise RuntimeError("h_full must be CUDA tensor.")
    if not kernel_chunk.is_cuda:
        raise RuntimeError("kernel_chunk must be CUDA tensor.")
    if h_full.dim() != 3:
        raise RuntimeError(f"h_full must be [B,D,L], got {tuple(h_full.shape)}.")
    if kernel_chunk.dim() != 4:
        raise RuntimeError(f"kernel_chunk must be [B,K,N,T], got {tuple(kernel_chunk.shape)}.")
    B, _, L = h_full.shape
    Bk, K, _, T = kernel_chunk.shape
    if B != Bk:
        raise RuntimeError(f"B mismatch: h_full={B}, kernel_chunk={Bk}.")
    if T <= 0:
        raise RuntimeError("T must be positive.")
    if K <= 0:
        raise RuntimeError("K must be positive.")
    if t_offset < 0:
        raise RuntimeError("t_offset must be non-negative.")
    if t_offset + T > L:
        raise RuntimeError(
            f"t_offset + T must be <= L, got t_offset={t_offset}, T={T}, L={L}.")
    if h_full.dtype not in _DTYPES:
        raise RuntimeError(f"Unsupported dtype: {h_full.dtype}.")
    if kernel_chunk.dtype != h_full.dtype:
        raise RuntimeError("kernel_chunk dtype must equal h_full dtype.")


# ---------------------------------------------------------------------------------------
# autograd
# ---------------------------------------------------------------------------------------
class FusedDynamicConvChunkFunction(torch.autograd.Function):
    """Fused dynamic conv over a time chunk starting at ``t_offset`` of ``h_full``.

    Saves (h_full, kernel_chunk, kernel_mix); the backward returns grad_h_full at the
    full ``[B,D,L]`` shape (zero outside the chunk's receptive range), grad_kernel_chunk
    ``[B,K,N,T]`` and grad_kernel_mix ``[D,N]``.
    """

    @staticmethod
    def forward(ctx, h_full, kernel_chunk, kernel_mix, t_offset: int, dilation: int = 1):
        t_offset, dilation = int(t_offset), int(dilation)
        _check_forward_inputs(h_full, kernel_chunk, kernel_mix, t_offset, dilation)
        h_c, k_c, m_c = h_full.contiguous(), kernel_chunk.contiguous(), kernel_mix.contiguous()
        out = _EXT.forward_chunk(h_c, k_c, m_c, t_offset, dilation)
        ctx.save_for_backward(h_c, k_c, m_c)
        ctx.t_offset, ctx.dilation = t_offset, dilation
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if grad_out is None:
            return None, None, None, None, None
        h_full, kernel_chunk, kernel_mix = ctx.saved_tensors
        gh, gk, gm = _EXT.backward_chunk(grad_out.contiguous(), h_full, kernel_chunk, kernel_mix,
                                         ctx.t_offset, ctx.dilation)
        return gh, gk, gm, None, None


def fused_dynamic_conv_chunk(h_full, kernel_chunk, kernel_mix, t_offset: int,
                             dilation: int = 1) -> torch.Tensor:
    return FusedDynamicConvChunkFunction.apply(h_full, kernel_chunk, kernel_mix, int(t_offset),
                                               int(dilation))


def fused_dynamic_conv(h, kernel, kernel_mix, dilation: int = 1) -> torch.Tensor:
    return fused_dynamic_conv_chunk(h_full=h, kernel_chunk=kernel, kernel_mix=kernel_mix,
                                    t_offset=0, dilation=int(dilation))


class FusedDynamicConvFunction(torch.autograd.Function):
    """Whole-sequence form (t_offset = 0); autograd flows through the chunk function."""

    @staticmethod
    def forward(ctx, h, kernel, kernel_mix, dilation: int = 1):
        return fused_dynamic_conv_chunk(h_full=h, kernel_chunk=kernel, kernel_mix=kernel_mix,
                                        t_offset=0, dilation=int(dilation))

    @staticmethod
    def backward(ctx, grad_out):
        raise RuntimeError(
            "Internal error: FusedDynamicConvFunction should not receive backward directly.")


# ---------------------------------------------------------------------------------------
# plan warmup / cache helpers (reference :269-562)
# ---------------------------------------------------------------------------------------
def _positive_repeat(repeat) -> int:
    repeat = int(repeat)
    if repeat <= 0:
        raise RuntimeError("repeat must be positive.")
    return repeat


def fused_dynamic_conv_forward_warmup_chunk(h_full, kernel_chunk, kernel_mix, t_offset: int,
                                            dilation: int = 1, repeat: int = 3) -> int:
    t_offset, dilation, repeat = int(t_offset), int(dilation), _positive_repeat(repeat)
    _check_forward_inputs(h_full, kernel_chunk, kernel_mix, t_offset, dilation)
    return int(_EXT.forward_chunk_warmup(h_full.contiguous(), kernel_chunk.contiguous(),
                                         kernel_mix.contiguous(), t_offset, dilation, repeat))


def fused_dynamic_conv_forward_warmup(h, kernel, kernel_mix, dilation: int = 1,
                                      repeat: int = 3) -> int:
    return fused_dynamic_conv_forward_warmup_chunk(h_full=h, kernel_chunk=kernel,
                                                   kernel_mix=kernel_mix, t_offset=0,
                                                   dilation=int(dilation), repeat=int(repeat))


def fused_dynamic_conv_forward_cached_plan_chunk(h_full, kernel_chunk, kernel_mix,
                                                 t_offset: int, dilation: int = 1) -> int:
    t_offset, dilation = int(t_offset), int(dilation)
    _check_forward_inputs(h_full, kernel_chunk, kernel_mix, t_offset, dilation)
    return int(_EXT.forward_chunk_cached_plan(h_full.contiguous(), kernel_chunk.contiguous(),
                                              kernel_mix.contiguous(), t_offset, dilation))


def fused_dynamic_conv_forward_cached_plan(h, kernel, kernel_mix, dilation: int = 1) -> int:
    return fused_dynamic_conv_forward_cached_plan_chunk(h_full=h, kernel_chunk=kernel,
                                                        kernel_mix=kernel_mix, t_offset=0,
                                                        dilation=int(dilation))


def fused_dynamic_conv_forward_clear_warmup_cache() -> None:
    _EXT.forward_chunk_clear_warmup_cache()


def fused_dynamic_conv_forward_plan_name(plan_id: int) -> str:
    return str(_EXT.forward_plan_name(int(plan_id)))


def fused_dynamic_conv_backward_warmup_chunk(grad_out, h_full, kernel_chunk, kernel_mix,
                                             t_offset: int, dilation: int = 1,
                                             repeat: int = 3) -> int:
    t_offset, dilation, repeat = int(t_offset), int(dilation), _positive_repeat(repeat)
    _check_backward_inputs(grad_out, h_full, kernel_chunk, kernel_mix, t_offset, dilation)
    return int(_EXT.backward_chunk_warmup(grad_out.contiguous(), h_full.contiguous(),
                                          kernel_chunk.contiguous(), kernel_mix.contiguous(),
                                          t_offset, dilation, repeat))


def fused_dynamic_conv_backward_warmup(grad_out, h, kernel, kernel_mix, dilation: int = 1,
                                       repeat: int = 3) -> int:
    return fused_dynamic_conv_backward_warmup_chunk(grad_out=grad_out, h_full=h,
                                                    kernel_chunk=kernel, kernel_mix=kernel_mix,
                                                    t_offset=0, dilation=int(dilation),
                                                    repeat=int(repeat))


def fused_dynamic_conv_backward_cached_plan_chunk(h_full, kernel_chunk, t_offset: int,
                                                  dilation: int = 1) -> int:
    t_offset, dilation = int(t_offset), int(dilation)
    _check_backward_plan_inputs(h_full, kernel_chunk, t_offset, dilation)
    return int(_EXT.backward_chunk_cached_plan(h_full.contiguous(), kernel_chunk.contiguous(),
                                               t_offset, dilation))


def fused_dynamic_conv_backward_cached_plan(h, kernel, dilation: int = 1) -> int:
    return fused_dynamic_conv_backward_cached_plan_chunk(h_full=h, kernel_chunk=kernel,
                                                         t_offset=0, dilation=int(dilation))


def fused_dynamic_conv_backward_clear_warmup_cache() -> None:
    _EXT.backward_chunk_clear_warmup_cache()


def fused_dynamic_conv_backward_plan_name(plan_id: int) -> str:
    return str(_EXT.backward_plan_name(int(plan_id)))


# ---------------------------------------------------------------------------------------
# modules (reference :592-838)
# ---------------------------------------------------------------------------------------
class FusedDynamicConvChunk1d(nn.Module):
    """Owns the basis ``kernel_mix[D,N]`` (init N(0, init_scale)) and an optional bias[D]."""

    def __init__(self, embed_dim: int, num_kernels: int, init_scale: float = 0.02,
                 use_bias: bool = False, dtype=None, device=None):
        super().__init__()
        self.embed_dim = int(embed_dim)
        self.num_kernels = int(num_kernels)
        self.init_scale = float(init_scale)
        self.use_bias = bool(use_bias)
        if self.embed_dim <= 0:
            raise ValueError("embed_dim must be positive.")
        if self.num_kernels <= 0:
            raise ValueError("num_kernels must be positive.")
        kw = {"dtype": dtype, "device": device}
        self.kernel_mix = nn.Parameter(torch.empty(self.embed_dim, self.num_kernels, **kw))
        nn.init.normal_(self.kernel_mix, mean=0.0, std=self.init_scale)
        if self.use_bias:
            self.bias = nn.Parameter(torch.zeros(self.embed_dim, **kw))
        else:
            self.register_parameter("bias", None)

    def _mix_as(self, h_full):
        m = self.kernel_mix
        return m if m.dtype == h_full.dtype else m.to(dtype=h_full.dtype)

    def warmup_forward(self, h_full, kernel_chunk, t_offset: int, dilation: int = 1,
                       repeat: int = 3) -> int:
        return fused_dynamic_conv_forward_warmup_chunk(
            h_full=h_full, kernel_chunk=kernel_chunk, kernel_mix=self._mix_as(h_full),
            t_offset=int(t_offset), dilation=int(dilation), repeat=int(repeat))

    def cached_forward_plan(self, h_full, kernel_chunk, t_offset: int, dilation: int = 1) -> int:
        return fused_dynamic_conv_forward_cached_plan_chunk(
            h_full=h_full, kernel_chunk=kernel_chunk, kernel_mix=self._mix_as(h_full),
            t_offset=int(t_offset), dilation=int(dilation))

    def warmup_backward(self, grad_out, h_full, kernel_chunk, t_offset: int, dilation: int = 1,
                        repeat: int = 3) -> int:
        return fused_dynamic_conv_backward_warmup_chunk(
            grad_out=grad_out, h_full=h_full, kernel_chunk=kernel_chunk,
            kernel_mix=self._mix_as(h_full), t_offset=int(t_offset), dilation=int(dilation),
            repeat=int(repeat))

    def cached_backward_plan(self, h_full, kernel_chunk, t_offset: int, dilation: int = 1) -> int:
        return fused_dynamic_conv_backward_cached_plan_chunk(
            h_full=h_full, kernel_chunk=kernel_chunk, t_offset=int(t_offset),
            dilation=int(dilation))

    def forward(self, h_full, kernel_chunk, t_offset: int, dilation: int = 1) -> torch.Tensor:
        out = fused_dynamic_conv_chunk(h_full=h_full, kernel_chunk=kernel_chunk,
                                       kernel_mix=self._mix_as(h_full), t_offset=int(t_offset),
                                       dilation=int(dilation))
        if self.bias is not None:
            out = out + self.bias.to(dtype=out.dtype, device=out.device).view(1, -1, 1)
        return out


class FusedDynamicConv1d(FusedDynamicConvChunk1d):
    """Whole-sequence module: ``t_offset`` is always 0."""

    def warmup_forward(self, h, kernel, dilation: int = 1, repeat: int = 3) -> int:
        return super().warmup_forward(h_full=h, kernel_chunk=kernel, t_offset=0,
                                      dilation=int(dilation), repeat=int(repeat))

    def cached_forward_plan(self, h, kernel, dilation: int = 1) -> int:
        return super().cached_forward_plan(h_full=h, kernel_chunk=kernel, t_offset=0,
                                           dilation=int(dilation))

    def warmup_backward(self, grad_out, h, kernel, dilation: int = 1, repeat: int = 3) -> int:
        return super().warmup_backward(grad_out=grad_out, h_full=h, kernel_chunk=kernel,
                                       t_offset=0, dilation=int(dilation), repeat=int(repeat))

    def cached_backward_plan(self, h, kernel, dilation: int = 1) -> int:
        return super().cached_backward_plan(h_full=h, kernel_chunk=kernel, t_offset=0,
                                            dilation=int(dilation))

    def forward(self, h, kernel, dilation: int = 1) -> torch.Tensor:
        return super().forward(h_full=h, kernel_chunk=kernel, t_offset=0, dilation=int(dilation))
