"""Fused source conv: depthwise causal conv -> bias -> exact GELU -> static mix.

Same public names, plan constants, signatures, defaults and error messages as the
reference's ``cuda_ops/fused_source_conv_mixed.py`` (adjfangjiawei/DUDyConv); the ops
are ``torch.ops.fused_source_conv_mixed.*``, registered by the in-tree ``cuda_ops_ext``
binding over ``libdudyconv_b200.so``.

Layout and semantics (reference ``cuda_ops/fused_source_conv_mixed_plans.h:7-44``)::

    x_norm [B,D,L]  weight [D,C,S]  bias [D,C] or None  mix_weight [D,C]  mix_bias [D]
    z[b,d,c,t]  = bias[d,c] + sum_j x_norm[b,d, off+t-dilation*(S-1-j)] * weight[d,c,j]
    out[b,d,t]  = mix_bias[d] + sum_c GELU(z[b,d,c,t]) * mix_weight[d,c]     -> [B,D,T]

Every legal plan id runs this library's kernels; plan ids select tiling only.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import load_extension

_CUDA_OPS_EXT = load_extension()  # registers TORCH_LIBRARY(fused_source_conv_mixed)
_FSCM_OPS = torch.ops.fused_source_conv_mixed

FORWARD_PLAN_GENERIC = 0
FORWARD_PLAN_C8S3 = 1
FORWARD_PLAN_C32S3 = 2
FORWARD_PLAN_D256C16S3 = 3
FORWARD_PLAN_GENERIC_NO_BOUNDARY = 100
FORWARD_PLAN_C8S3_NO_BOUNDARY = 101
FORWARD_PLAN_C32S3_NO_BOUNDARY = 102
FORWARD_PLAN_D256C16S3_NO_BOUNDARY = 103

BACKWARD_PLAN_ATOMIC = 0
BACKWARD_PLAN_PER_D_REDUCE = 1
BACKWARD_PLAN_GATHER_X = 2

_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def _empty_bias_like_input(x_norm: torch.Tensor) -> torch.Tensor:
    return torch.empty(0, device=x_norm.device, dtype=x_norm.dtype)


def _has_bias(bias) -> bool:
    return bias is not None and bias.numel() > 0


# ---------------------------------------------------------------------------------------
# checks (reference cuda_ops/fused_source_conv_mixed.py:38-226)
# ---------------------------------------------------------------------------------------
def _check_source_conv_mixed_forward_inputs(x_norm, weight, bias, mix_weight, mix_bias, off,
                                            T, dilation) -> None:
    off, T, dilation = int(off), int(T), int(dilation)
    for name, t in (("x_norm", x_norm), ("weight", weight)):
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be CUDA tensor.")
    if _has_bias(bias) and not bias.is_cuda:
        raise RuntimeError("bias must be CUDA tensor when provided.")
    for name, t in (("mix_weight", mix_weight), ("mix_bias", mix_bias)):
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be CUDA tensor.")
    if x_norm.dim() != 3:
        raise RuntimeError(f"x_norm must be [B,D,L], got {tuple(x_norm.shape)}.")
    if weight.dim() != 3:
        raise RuntimeError(f"weight must be [D,C,S], got {tuple(weight.shape)}.")
    if mix_weight.dim() != 2:
        raise RuntimeError(f"mix_weight must be [D,C], got {tuple(mix_weight.shape)}.")
    if mix_bias.dim() != 1:
        raise RuntimeError(f"mix_bias must be [D], got {tuple(mix_bias.shape)}.")
    B, D, L = x_norm.shape
    Dw, C, S = weight.shape
    for name, v in (("B", B), ("D", D), ("L", L), ("C", C), ("S", S)):
        if v <= 0:
            raise RuntimeError(f"{name} must be positive.")
    if Dw != D:
        raise RuntimeError(f"weight D mismatch: weight={Dw}, x_norm={D}.")
    if mix_weight.shape[0] != D:
        raise RuntimeError(f"mix_weight D mismatch: mix_weight={mix_weight.shape[0]}, x_norm={D}.")
    if mix_weight.shape[1] != C:
        raise RuntimeError(f"mix_weight C mismatch: mix_weight={mix_weight.shape[1]}, weight={C}.")
    if mix_bias.shape[0] != D:
        raise RuntimeError(f"mix_bias D mismatch: mix_bias={mix_bias.shape[0]}, x_norm={D}.")
    if _has_bias(bias):
        if bias.dim() != 2:
            raise RuntimeError(f"bias must be [D,C], got {tuple(bias.shape)}.")
        if bias.shape[0] != D:
            raise RuntimeError(f"bias D mismatch: bias={bias.shape[0]}, x_norm={D}.")
        if bias.shape[1] != C:
            raise RuntimeError(f"bias C mismatch: bias={bias.shape[1]}, weight={C}.")
    if off < 0:
        raise RuntimeError("off must be non-negative.")
    if T <= 0:
        raise RuntimeError("T must be positive.")
    if off + T > L:
        raise RuntimeError(f"off + T must be <= L, got off={off}, T={T}, L={L}.")
    if dilation <= 0:
        raise RuntimeError("dilation must be positive.")
    if x_norm.dtype not in _DTYPES:
        raise RuntimeError(f"Unsupported dtype: {x_norm.dtype}.")
    for name, t in (("weight", weight), ("mix_weight", mix_weight), ("mix_bias", mix_bias)):
        if t.dtype != x_norm.dtype:
            raise RuntimeError(f"{name} dtype must equal x_norm dtype.")
    if _has_bias(bias) and bias.dtype != x_norm.dtype:
        raise RuntimeError("bias dtype must equal x_norm dtype.")


def _check_source_conv_mixed_backward_inputs(grad_out, x_norm, weight, bias, mix_weight,
                                             mix_bias, off, T, dilation) -> None:
    _check_source_conv_mixed_forward_inputs(x_norm, weight, bias, mix_weight, mix_bias, off, T,
                                            dilation)
    if not grad_out.is_cuda:
        raise RuntimeError("grad_out must be CUDA tensor.")
    if grad_out.dim() != 3:
        raise RuntimeError(f"grad_out must be [B,D,T], got {tuple(grad_out.shape)}.")
    B, D, _ = x_norm.shape
    if grad_out.shape[0] != B:
        raise RuntimeError(f"grad_out B mismatch: grad_out={grad_out.shape[0]}, x_norm={B}.")
    if grad_out.shape[1] != D:
        raise RuntimeError(f"grad_out D mismatch: grad_out={grad_out.shape[1]}, x_norm={D}.")
    if grad_out.shape[2] != int(T):
        raise RuntimeError(f"grad_out T mismatch: grad_out={grad_out.shape[2]}, T={int(T)}.")
    if grad_out.dtype != x_norm.dtype:
        raise RuntimeError("grad_out dtype must equal x_norm dtype.")


def _as_bias_tensor(x_norm, bias):
    return _empty_bias_like_input(x_norm) if bias is None else bias


def _prep(x_norm, weight, bias, mix_weight, mix_bias):
    x_c = x_norm.contiguous()
    return (x_c, weight.contiguous(), _as_bias_tensor(x_c, bias).contiguous(),
            mix_weight.contiguous(), mix_bias.contiguous())


def _grads_out(grads, bias):
    return grads[0], grads[1], (grads[2] if bias is not None else None), grads[3], grads[4]


# ---------------------------------------------------------------------------------------
# autograd
# ---------------------------------------------------------------------------------------
class FusedSourceConvMixedFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_norm, weight, bias, mix_weight, mix_bias, off: int, T: int,
                dilation: int = 1):
        off, T, dilation = int(off), int(T), int(dilation)
        _check_source_conv_mixed_forward_inputs(x_norm, weight, bias, mix_weight, mix_bias, off,
                                                T, dilation)
        args = _prep(x_norm, weight, bias, mix_weight, mix_bias)
        out = _FSCM_OPS.forward(*args, off, T, dilation)
        ctx.save_for_backward(*args)
        ctx.has_bias = _has_bias(bias)
        ctx.off, ctx.T, ctx.dilation = off, T, dilation
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if grad_out is None:
            return (None,) * 8
        x_norm, weight, bias, mix_weight, mix_bias = ctx.saved_tensors
        g = _FSCM_OPS.backward(grad_out.contiguous(), x_norm, weight, bias, mix_weight, mix_bias,
                               ctx.off, ctx.T, ctx.dilation)
        return g[0], g[1], (g[2] if ctx.has_bias else None), g[3], g[4], None, None, None


def fused_source_conv_mixed(x_norm, weight, bias, mix_weight, mix_bias, off: int, T: int,
                            dilation: int = 1) -> torch.Tensor:
    return FusedSourceConvMixedFunction.apply(x_norm, weight, bias, mix_weight, mix_bias,
                                              int(off), int(T), int(dilation))


# ---------------------------------------------------------------------------------------
# functional entries (reference :376-819)
# ---------------------------------------------------------------------------------------
def fused_source_conv_mixed_forward(x_norm, weight, bias, mix_weight, mix_bias, off: int,
                                    T: int, dilation: int = 1) -> torch.Tensor:
    _check_source_conv_mixed_forward_inputs(x_norm, weight, bias, mix_weight, mix_bias, off, T,
                                            dilation)
    return _FSCM_OPS.forward(*_prep(x_norm, weight, bias, mix_weight, mix_bias), int(off), int(T),
                             int(dilation))


def fused_source_conv_mixed_forward_plan(x_norm, weight, bias, mix_weight, mix_bias, off: int,
                                         T: int, dilation: int, plan: int) -> torch.Tensor:
    _check_source_conv_mixed_forward_inputs(x_norm, weight, bias, mix_weight, mix_bias, off, T,
                                            dilation)
    return _FSCM_OPS.forward_plan(*_prep(x_norm, weight, bias, mix_weight, mix_bias), int(off),
                                  int(T), int(dilation), int(plan))


def fused_source_conv_mixed_forward_cached_plan(x_norm, weight, bias, mix_weight, mix_bias,
                                                off: int, T: int, dilation: int,
                                                cached_plan: int) -> torch.Tensor:
    _check_source_conv_mixed_forward_inputs(x_norm, weight, bias, mix_weight, mix_bias, off, T,
                                            dilation)
    return _FSCM_OPS.forward_cached_plan(*_prep(x_norm, weight, bias, mix_weight, mix_bias),
                                         int(off), int(T), int(dilation), int(cached_plan))


def _check_iters(warmup_iters, bench_iters) -> None:
    if warmup_iters < 0:
        raise RuntimeError("warmup_iters must be >= 0.")
    if bench_iters <= 0:
        raise RuntimeError("bench_iters must be positive.")


def fused_source_conv_mixed_forward_warmup(x_norm, weight, bias, mix_weight, mix_bias, off: int,
                                           T: int, dilation: int = 1, warmup_iters: int = 2,
                                           bench_iters: int = 5) -> int:
    _check_iters(warmup_iters, bench_iters)
    _check_source_conv_mixed_forward_inputs(x_norm, weight, bias, mix_weight, mix_bias, off, T,
                                            dilation)
    return int(_FSCM_OPS.forward_warmup(*_prep(x_norm, weight, bias, mix_weight, mix_bias),
                                        int(off), int(T), int(dilation), int(warmup_iters),
                                        int(bench_iters)))


def fused_source_conv_mixed_backward(grad_out, x_norm, weight, bias, mix_weight, mix_bias,
                                     off: int, T: int, dilation: int = 1):
    _check_source_conv_mixed_backward_inputs(grad_out, x_norm, weight, bias, mix_weight,
                                             mix_bias, off, T, dilation)
    g = _FSCM_OPS.backward(grad_out.contiguous(), *_prep(x_norm, weight, bias, mix_weight,
                                                         mix_bias), int(off), int(T),
                           int(dilation))
    return _grads_out(g, bias)


def fused_source_conv_mixed_backward_plan(grad_out, x_norm, weight, bias, mix_weight, mix_bias,
                                          off: int, T: int, dilation: int, plan: int,
                                          tile_t: int):
    _check_source_conv_mixed_backward_inputs(grad_out, x_norm, weight, bias, mix_weight,
                                             mix_bias, off, T, dilation)
    g = _FSCM_OPS.backward_plan(grad_out.contiguous(), *_prep(x_norm, weight, bias, mix_weight,
                                                              mix_bias), int(off), int(T),
                                int(dilation), int(plan), int(tile_t))
    return _grads_out(g, bias)


def fused_source_conv_mixed_backward_cached_plan(grad_out, x_norm, weight, bias, mix_weight,
                                                 mix_bias, off: int, T: int, dilation: int,
                                                 cached_plan: int):
    _check_source_conv_mixed_backward_inputs(grad_out, x_norm, weight, bias, mix_weight,
                                             mix_bias, off, T, dilation)
    g = _FSCM_OPS.backward_cached_plan(grad_out.contiguous(), *_prep(x_norm, weight, bias,
                                                                     mix_weight, mix_bias),
                                       int(off), int(T), int(dilation), int(cached_plan))
    return _grads_out(g, bias)


def fused_source_conv_mixed_backward_warmup(grad_out, x_norm, weight, bias, mix_weight, mix_bias,
                                            off: int, T: int, dilation: int = 1,
                                            warmup_iters: int = 2, bench_iters: int = 5) -> int:
    _check_iters(warmup_iters, bench_iters)
    _check_source_conv_mixed_backward_inputs(grad_out, x_norm, weight, bias, mix_weight,
                                             mix_bias, off, T, dilation)
    return int(_FSCM_OPS.backward_warmup(grad_out.contiguous(),
                                         *_prep(x_norm, weight, bias, mix_weight, mix_bias),
                                         int(off), int(T), int(dilation), int(warmup_iters),
                                         int(bench_iters)))


def fused_source_conv_mixed_backward_pack_cached_plan(plan: int, tile_t: int) -> int:
    return int(_FSCM_OPS.backward_pack_cached_plan(int(plan), int(tile_t)))


def fused_source_conv_mixed_backward_cached_plan_get_plan(cached_plan: int) -> int:
    return int(_FSCM_OPS.backward_cached_plan_get_plan(int(cached_plan)))


def fused_source_conv_mixed_backward_cached_plan_get_tile_t(cached_plan: int) -> int:
    return int(_FSCM_OPS.backward_cached_plan_get_tile_t(int(cached_plan)))


_FORWARD_NAMES = {
    FORWARD_PLAN_GENERIC: "Generic", FORWARD_PLAN_C8S3: "C8S3", FORWARD_PLAN_C32S3: "C32S3",
    FORWARD_PLAN_D256C16S3: "D256C16S3", FORWARD_PLAN_GENERIC_NO_BOUNDARY: "GenericNoBoundary",
    FORWARD_PLAN_C8S3_NO_BOUNDARY: "C8S3NoBoundary",
    FORWARD_PLAN_C32S3_NO_BOUNDARY: "C32S3NoBoundary",
    FORWARD_PLAN_D256C16S3_NO_BOUNDARY: "D256C16S3NoBoundary",
}
_BACKWARD_NAMES = {BACKWARD_PLAN_ATOMIC: "Atomic", BACKWARD_PLAN_PER_D_REDUCE: "PerDReduce",
                   BACKWARD_PLAN_GATHER_X: "GatherX"}


def fused_source_conv_mixed_forward_plan_name(plan: int) -> str:
    plan = int(plan)
    return _FORWARD_NAMES.get(plan, f"unknown_forward_plan_{plan}")


def fused_source_conv_mixed_backward_plan_name(plan: int) -> str:
    plan = int(plan)
    return _BACKWARD_NAMES.get(plan, f"unknown_backward_plan_{plan}")


# ---------------------------------------------------------------------------------------
# modules (reference :822-1090)
# ---------------------------------------------------------------------------------------
class FusedSourceConvMixedChunk1d(nn.Module):
    def __init__(self, embed_dim: int, source_channels: int, kernel_size: int,
                 init_scale: float = 0.02, use_bias: bool = True, dtype=None, device=None):
        super().__init__()
        self.embed_dim = int(embed_dim)
        self.source_channels = int(source_channels)
        self.kernel_size = int(kernel_size)
        self.init_scale = float(init_scale)
        self.use_bias = bool(use_bias)
        if self.embed_dim <= 0:
            raise ValueError("embed_dim must be positive.")
        if self.source_channels <= 0:
            raise ValueError("source_channels must be positive.")
        if self.kernel_size <= 0:
            raise ValueError("kernel_size must be positive.")
        kw = {"dtype": dtype, "device": device}
        D, C, S = self.embed_dim, self.source_channels, self.kernel_size
        self.weight = nn.Parameter(torch.empty(D, C, S, **kw))
        self.mix_weight = nn.Parameter(torch.empty(D, C, **kw))
        self.mix_bias = nn.Parameter(torch.zeros(D, **kw))
        if self.use_bias:
            self.bias = nn.Parameter(torch.zeros(D, C, **kw))
        else:
            self.register_parameter("bias", None)
        nn.init.normal_(self.weight, mean=0.0, std=self.init_scale)
        nn.init.normal_(self.mix_weight, mean=0.0, std=self.init_scale)

    def _params_as(self, x_norm):
        def cast(p):
            return p if p is None or p.dtype == x_norm.dtype else p.to(dtype=x_norm.dtype)
        return cast(self.weight), cast(self.bias), cast(self.mix_weight), cast(self.mix_bias)

    def warmup_forward(self, x_norm, off: int, T: int, dilation: int = 1, warmup_iters: int = 2,
                       bench_iters: int = 5) -> int:
        w, b, mw, mb = self._params_as(x_norm)
        return fused_source_conv_mixed_forward_warmup(
            x_norm=x_norm, weight=w, bias=b, mix_weight=mw, mix_bias=mb, off=int(off), T=int(T),
            dilation=int(dilation), warmup_iters=int(warmup_iters), bench_iters=int(bench_iters))

    def warmup_backward(self, grad_out, x_norm, off: int, T: int, dilation: int = 1,
                        warmup_iters: int = 2, bench_iters: int = 5) -> int:
        w, b, mw, mb = self._params_as(x_norm)
        return fused_source_conv_mixed_backward_warmup(
            grad_out=grad_out, x_norm=x_norm, weight=w, bias=b, mix_weight=mw, mix_bias=mb,
            off=int(off), T=int(T), dilation=int(dilation), warmup_iters=int(warmup_iters),
            bench_iters=int(bench_iters))

    def forward(self, x_norm, off: int, T: int, dilation: int = 1) -> torch.Tensor:
        w, b, mw, mb = self._params_as(x_norm)
        return fused_source_conv_mixed(x_norm=x_norm, weight=w, bias=b, mix_weight=mw,
                                       mix_bias=mb, off=int(off), T=int(T),
                                       dilation=int(dilation))


class FusedSourceConvMixed1d(FusedSourceConvMixedChunk1d):
    """Whole-sequence module: off = 0 and T = L."""

    def warmup_forward(self, x_norm, dilation: int = 1, warmup_iters: int = 2,
                       bench_iters: int = 5) -> int:
        return super().warmup_forward(x_norm=x_norm, off=0, T=int(x_norm.shape[2]),
                                      dilation=int(dilation), warmup_iters=int(warmup_iters),
                                      bench_iters=int(bench_iters))

    def warmup_backward(self, grad_out, x_norm, dilation: int = 1, warmup_iters: int = 2,
                        bench_iters: int = 5) -> int:
        return super().warmup_backward(grad_out=grad_out, x_norm=x_norm, off=0,
                                       T=int(x_norm.shape[2]), dilation=int(dilation),
                                       warmup_iters=int(warmup_iters),
                                       bench_iters=int(bench_iters))

    def forward(self, x_norm, dilation: int = 1) -> torch.Tensor:
        return super().forward(x_norm=x_norm, off=0, T=int(x_norm.shape[2]),
                               dilation=int(dilation))
