"""Oracle for ``fused_dynamic_conv_chunk`` (test infrastructure only).

Semantics (adjfangjiawei/DUDyConv ``cuda_ops/fused_dynamic_conv.py:7-31``,
``cuda_ops/fused_dynamic_conv_plans.h:8-28``,
``test_fused_dynamic_conv_against_reference.py:91-189``)::

    h    [B, D, L]     kc [B, K, N, T]     mix [D, N]
    out[b, d, t] = sum_kk sum_n h[b, d, off + t - kk*dil] * kc[b, kk, n, t] * mix[d, n]

Taps whose source index is negative contribute nothing (causal zero padding);
``off + T <= L`` is a precondition, so the source never runs past ``L``.

Backward (the autograd of the formula above; the reference returns
``grad_h`` at full ``[B, D, L]``, zero outside ``[off-(K-1)*dil, off+T)``)::

    G_kk[b, d, t]        = go[b, d, t] * h[b, d, off + t - kk*dil]
    grad_kc[b, kk, n, t] = sum_d mix[d, n] * G_kk[b, d, t]
    grad_mix[d, n]       = sum_{b, kk, t} G_kk[b, d, t] * kc[b, kk, n, t]
    grad_h[b, d, off + t - kk*dil] += go[b, d, t] * W_kk[b, d, t],
    W_kk[b, d, t]        = sum_n mix[d, n] * kc[b, kk, n, t]
"""

from __future__ import annotations

import numpy as np


def _tap_window(off: int, T: int, kk: int, dil: int):
    """Destination range [t0, T) of tap kk and its source start in h.

    Mirrors the clipping in ``torch_reference_materialized_chunk``
    (``test_fused_dynamic_conv_against_reference.py:154-183``).
    """
    src0 = off - kk * dil
    t0 = 0
    if src0 < 0:
        t0 = -src0
        src0 = 0
    return t0, src0


def _check(h, kc, mix, off, dil):
    B, D, L = h.shape
    Bk, K, N, T = kc.shape
    assert B == Bk and mix.shape == (D, N)
    assert off >= 0 and dil > 0 and off + T <= L


def fdc_forward(h, kc, mix, off: int, dil: int = 1, dtype=np.float64):
    """out[B, D, T]; computed in ``dtype`` (float64 for parity, float32 for timing)."""
    _check(h, kc, mix, off, dil)
    h = np.asarray(h, dtype=dtype)
    kc = np.asarray(kc, dtype=dtype)
    mix = np.asarray(mix, dtype=dtype)
    B, D, L = h.shape
    _, K, N, T = kc.shape
    out = np.zeros((B, D, T), dtype=dtype)
    for kk in range(K):
        t0, src0 = _tap_window(off, T, kk, dil)
        if t0 >= T:
            continue
        # W_kk[b] = mix @ kc[b, kk]  -> [B, D, T - t0]
        w = np.matmul(mix[None, :, :], kc[:, kk, :, t0:])
        out[:, :, t0:] += w * h[:, :, src0:src0 + (T - t0)]
    return out


def fdc_backward(go, h, kc, mix, off: int, dil: int = 1, dtype=np.float64):
    """Returns (grad_h [B,D,L], grad_kc [B,K,N,T], grad_mix [D,N])."""
    _check(h, kc, mix, off, dil)
    go = np.asarray(go, dtype=dtype)
    h = np.asarray(h, dtype=dtype)
    kc = np.asarray(kc, dtype=dtype)
    mix = np.asarray(mix, dtype=dtype)
    B, D, L = h.shape
    _, K, N, T = kc.shape
    assert go.shape == (B, D, T)
    grad_h = np.zeros((B, D, L), dtype=dtype)
    grad_kc = np.zeros((B, K, N, T), dtype=dtype)
    grad_mix = np.zeros((D, N), dtype=dtype)
    mix_t = np.ascontiguousarray(mix.T)
    for kk in range(K):
        t0, src0 = _tap_window(off, T, kk, dil)
        if t0 >= T:
            continue
        n_t = T - t0
        hs = h[:, :, src0:src0 + n_t]
        g = go[:, :, t0:] * hs                                   # G_kk  [B, D, n_t]
        grad_kc[:, kk, :, t0:] = np.matmul(mix_t[None], g)        # [B, N, n_t]
        kck = kc[:, kk, :, t0:]                                   # [B, N, n_t]
        grad_mix += np.einsum("bdt,bnt->dn", g, kck, optimize=True)
        w = np.matmul(mix[None], kck)                             # W_kk  [B, D, n_t]
        grad_h[:, :, src0:src0 + n_t] += go[:, :, t0:] * w
    return grad_h, grad_kc, grad_mix


def fdc_forward_backward_fp32(h, kc, mix, go, off: int, dil: int = 1):
    """One fwd+bwd pass in float32: the CPU baseline that ``bench.py`` times."""
    out = fdc_forward(h, kc, mix, off, dil, dtype=np.float32)
    grads = fdc_backward(go, h, kc, mix, off, dil, dtype=np.float32)
    return out, grads
