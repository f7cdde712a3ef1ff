"""Oracle for ``fused_source_conv_mixed`` (test infrastructure only).

Semantics (adjfangjiawei/DUDyConv ``cuda_ops/fused_source_conv_mixed_plans.h:7-44``,
``test_fused_source_conv_mixed.py:111-255``)::

    x [B, D, L]   weight [D, C, S]   bias [D, C] or None   mix_w [D, C]   mix_b [D]
    z[b, d, c, t] = bias[d, c] + sum_j x[b, d, off + t - dil*(S-1-j)] * weight[d, c, j]
    out[b, d, t]  = mix_b[d] + sum_c GELU(z[b, d, c, t]) * mix_w[d, c]

GELU is the exact (erf) form, ``F.gelu(approximate="none")``. Tap ``j = S-1``
is the current token; sources below index 0 read as zero.

Backward (autograd of the same formula)::

    gz[b,d,c,t]      = go[b,d,t] * mix_w[d,c] * GELU'(z)
    grad_mix_w[d,c]  = sum_{b,t} go * GELU(z)
    grad_mix_b[d]    = sum_{b,t} go
    grad_bias[d,c]   = sum_{b,t} gz
    grad_w[d,c,j]    = sum_{b,t} gz * x[b,d,src_j(t)]
    grad_x[b,d,src_j(t)] += sum_c gz[b,d,c,t] * weight[d,c,j]     (full [B,D,L])
"""

from __future__ import annotations

import numpy as np
from scipy.special import erf

_INV_SQRT2 = 0.7071067811865476
_INV_SQRT2PI = 0.3989422804014327


def gelu(z):
    return 0.5 * z * (1.0 + erf(z * _INV_SQRT2))


def gelu_grad(z):
    return 0.5 * (1.0 + erf(z * _INV_SQRT2)) + z * np.exp(-0.5 * z * z) * _INV_SQRT2PI


def _shifted(x, off, T, shift):
    """x[:, :, off + t - shift] for t in [0, T), zero where the index is negative."""
    B, D, L = x.shape
    out = np.zeros((B, D, T), dtype=x.dtype)
    src0 = off - shift
    t0 = max(0, -src0)
    if t0 < T:
        out[:, :, t0:] = x[:, :, src0 + t0:src0 + T]
    return out


def _z(x, weight, bias, off, T, dil):
    D, C, S = weight.shape
    B = x.shape[0]
    z = np.zeros((B, D, C, T), dtype=x.dtype)
    if bias is not None:
        z += bias[None, :, :, None]
    xs = [_shifted(x, off, T, dil * (S - 1 - j)) for j in range(S)]
    for j in range(S):
        z += xs[j][:, :, None, :] * weight[None, :, :, j, None]
    return z, xs


def fscm_forward(x, weight, bias, mix_w, mix_b, off: int, T: int, dil: int = 1,
                 dtype=np.float64):
    x = np.asarray(x, dtype=dtype)
    weight = np.asarray(weight, dtype=dtype)
    bias = None if bias is None or np.size(bias) == 0 else np.asarray(bias, dtype=dtype)
    mix_w = np.asarray(mix_w, dtype=dtype)
    mix_b = np.asarray(mix_b, dtype=dtype)
    assert off >= 0 and T > 0 and off + T <= x.shape[2] and dil > 0
    z, _ = _z(x, weight, bias, off, T, dil)
    return mix_b[None, :, None] + np.einsum("bdct,dc->bdt", gelu(z), mix_w)


def fscm_backward(go, x, weight, bias, mix_w, mix_b, off: int, T: int, dil: int = 1,
                  dtype=np.float64):
    """Returns (grad_x, grad_w, grad_bias or None, grad_mix_w, grad_mix_b)."""
    go = np.asarray(go, dtype=dtype)
    x = np.asarray(x, dtype=dtype)
    weight = np.asarray(weight, dtype=dtype)
    has_bias = bias is not None and np.size(bias) > 0
    bias = np.asarray(bias, dtype=dtype) if has_bias else None
    mix_w = np.asarray(mix_w, dtype=dtype)
    B, D, L = x.shape
    _, C, S = weight.shape
    z, xs = _z(x, weight, bias, off, T, dil)
    a = gelu(z)
    gz = go[:, :, None, :] * mix_w[None, :, :, None] * gelu_grad(z)
    grad_mix_w = np.einsum("bdt,bdct->dc", go, a)
    grad_mix_b = go.sum(axis=(0, 2))
    grad_bias = gz.sum(axis=(0, 3)) if has_bias else None
    grad_w = np.zeros((D, C, S), dtype=dtype)
    grad_x = np.zeros((B, D, L), dtype=dtype)
    for j in range(S):
        grad_w[:, :, j] = np.einsum("bdct,bdt->dc", gz, xs[j])
        contrib = np.einsum("bdct,dc->bdt", gz, weight[:, :, j])
        src0 = off - dil * (S - 1 - j)
        t0 = max(0, -src0)
        if t0 < T:
            grad_x[:, :, src0 + t0:src0 + T] += contrib[:, :, t0:]
    return grad_x, grad_w, grad_bias, grad_mix_w, grad_mix_b
