"""Oracle for the kernel generator's tail (test infrastructure only).

Restates ``StreamingKernelGenConv1d._logits_to_kernel``
(adjfangjiawei/DUDyConv ``backbone_dil_unshared.py:1821-1900``) and its autograd
backward in numpy float64::

    y  = softmax over k of logits.reshape(B, N, K, T)
    kc[b, kk, n, t] = y[b, n, K-1-kk, t]                     (flip K, permute)
    grad_logits[b, n*K+k, t] = y_k * (g_k - sum_j y_j g_j),  g_k = grad_kc[b, K-1-k, n, t]

Pinned by ``tests/golden/kgen_golden.npz`` (made from the reference's own method).
"""

from __future__ import annotations

import numpy as np


def logits_to_kernel(logits, N: int, K: int, dtype=np.float64):
    x = np.asarray(logits, dtype=dtype)
    B, M, T = x.shape
    assert M == N * K
    y = x.reshape(B, N, K, T)
    y = np.exp(y - y.max(axis=2, keepdims=True))
    y = y / y.sum(axis=2, keepdims=True)
    return np.ascontiguousarray(y[:, :, ::-1, :].transpose(0, 2, 1, 3))


def logits_to_kernel_backward(logits, grad_kc, N: int, K: int, dtype=np.float64):
    kc = logits_to_kernel(logits, N, K, dtype)
    g = np.asarray(grad_kc, dtype=dtype)
    dot = (kc * g).sum(axis=1, keepdims=True)                  # [B,1,N,T]
    gk = kc * (g - dot)                                        # [B,K,N,T] in tap order
    B, _, _, T = gk.shape
    return np.ascontiguousarray(gk[:, ::-1].transpose(0, 2, 1, 3).reshape(B, N * K, T))
