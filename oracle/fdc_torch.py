"""The dynamic-conv oracle in torch float64 (test infrastructure only).

The same restatement as ``oracle/fdc.py`` (adjfangjiawei/DUDyConv
``test_fused_dynamic_conv_against_reference.py:91-189``: the materialised formula and its
autograd backward), written with torch so it can run in float64 on whatever device holds
the inputs. The GPU parity tests use it to check BASELINE-size calls (B=16, T=4096) in
full, where the numpy oracle would take minutes; ``tests/test_oracle_golden.py`` pins it
against the numpy oracle and the golden fixtures on the CPU.

Nothing in the shipped library imports this module.
"""

from __future__ import annotations

import torch


def _windows(off: int, T: int, K: int, dil: int):
    """(kk, t0, src0) for every tap that reaches a token: destination tokens [t0, T) read
    h positions [src0, src0 + T - t0) (causal clipping of the materialised formula,
    ``test_fused_dynamic_conv_against_reference.py:154-183``)."""
    for kk in range(K):
        src0 = off - kk * dil
        t0 = 0
        if src0 < 0:
            t0, src0 = -src0, 0
        if t0 < T:
            yield kk, t0, src0


def fdc_forward_t(h, kc, mix, off: int, dil: int = 1):
    """out[B, D, T] in float64 on the inputs' device."""
    h, kc, mix = h.double(), kc.double(), mix.double()
    B, D, L = h.shape
    _, K, N, T = kc.shape
    out = torch.zeros(B, D, T, dtype=torch.float64, device=h.device)
    for kk, t0, src0 in _windows(off, T, K, dil):
        n = T - t0
        w = torch.matmul(mix, kc[:, kk, :, t0:])                   # W_kk [B, D, n]
        out[:, :, t0:] += w * h[:, :, src0:src0 + n]
    return out


def fdc_backward_t(go, h, kc, mix, off: int, dil: int = 1):
    """(grad_h [B,D,L], grad_kc [B,K,N,T], grad_mix [D,N]) in float64."""
    go, h, kc, mix = go.double(), h.double(), kc.double(), mix.double()
    B, D, L = h.shape
    _, K, N, T = kc.shape
    dev = h.device
    grad_h = torch.zeros(B, D, L, dtype=torch.float64, device=dev)
    grad_kc = torch.zeros(B, K, N, T, dtype=torch.float64, device=dev)
    grad_mix = torch.zeros(D, N, dtype=torch.float64, device=dev)
    mix_t = mix.t().contiguous()
    for kk, t0, src0 in _windows(off, T, K, dil):
        n = T - t0
        g = go[:, :, t0:] * h[:, :, src0:src0 + n]                 # G_kk [B, D, n]
        grad_kc[:, kk, :, t0:] = torch.matmul(mix_t, g)
        kck = kc[:, kk, :, t0:]
        grad_mix += torch.einsum("bdt,bnt->dn", g, kck)
        grad_h[:, :, src0:src0 + n] += go[:, :, t0:] * torch.matmul(mix, kck)
        del g
    return grad_h, grad_kc, grad_mix
