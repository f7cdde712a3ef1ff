"""Deterministic inputs for the golden fixtures.

The fixtures store only the case geometry and the reference's outputs; the
inputs are re-drawn here from a seed with numpy's PCG64 generator, rounded to
the case dtype (fp32 / fp16 / bf16, round-to-nearest-even) and returned as
exact float32 arrays. ``make_golden.py`` uses the same functions, so the
reference formulas and the tests see bit-identical inputs.
"""

from __future__ import annotations

import numpy as np


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` and return them as exact float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "fp32":
        return x.copy()
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        # round to nearest even on the upper 16 bits
        lsb = (u >> 16) & 1
        u = (u + 0x7FFF + lsb) & 0xFFFF0000
        return u.astype(np.uint32).view(np.float32)
    raise ValueError(dtype)


def draw(rng: np.random.Generator, shape, std: float, dtype: str) -> np.ndarray:
    x = rng.standard_normal(size=shape, dtype=np.float32) * np.float32(std)
    return round_to(x, dtype)


def fdc_inputs(meta, dtype: str, dist: str, seed: int):
    """(h, kc, mix, go) for a dynamic-conv case; meta = (B, D, L, T, N, K, off, dil)."""
    B, D, L, T, N, K, off, dil = (int(v) for v in meta)
    rng = np.random.Generator(np.random.PCG64(seed))
    if dist == "ref":
        # the reference tests scale every randn leaf by 0.1
        # (test_fused_dynamic_conv_against_reference.py:41-68,380-417)
        s_h = s_kc = s_mix = s_go = 0.1
    else:
        # BASELINE distributions: h, go ~ N(0,1); kc ~ N(0,1/N); mix ~ N(0,1/3)
        s_h, s_kc, s_mix, s_go = 1.0, (1.0 / N) ** 0.5, (1.0 / 3.0) ** 0.5, 1.0
    h = draw(rng, (B, D, L), s_h, dtype)
    kc = draw(rng, (B, K, N, T), s_kc, dtype)
    mix = draw(rng, (D, N), s_mix, dtype)
    go = draw(rng, (B, D, T), s_go, dtype)
    return h, kc, mix, go


def fscm_inputs(meta, dtype: str, seed: int):
    """(x, weight, bias or None, mix_w, mix_b, go); meta = (B, D, L, T, C, S, off, dil, bias)."""
    B, D, L, T, C, S, off, dil, use_bias = (int(v) for v in meta)
    rng = np.random.Generator(np.random.PCG64(seed))
    x = draw(rng, (B, D, L), 0.1, dtype)
    w = draw(rng, (D, C, S), 0.1, dtype)
    bias = draw(rng, (D, C), 0.1, dtype) if use_bias else None
    mw = draw(rng, (D, C), 0.1, dtype)
    mb = draw(rng, (D,), 0.1, dtype)
    go = draw(rng, (B, D, T), 0.1, dtype)
    return x, w, bias, mw, mb, go


def fscm_inputs_baseline(meta, dtype: str, seed: int):
    """Source-conv inputs at the benchmark distribution (config 3): x ~ N(0,1),
    weight ~ N(0,1/3), bias and mix_w ~ N(0,1/C), mix_b = 0, go ~ N(0,1).

    At this scale the pre-activations reach the tails of the erf-GELU (|z| of several
    units), which the reference tests' 0.1-scaled inputs never do."""
    B, D, L, T, C, S, off, dil, use_bias = (int(v) for v in meta)
    rng = np.random.Generator(np.random.PCG64(seed))
    x = draw(rng, (B, D, L), 1.0, dtype)
    w = draw(rng, (D, C, S), (1.0 / 3.0) ** 0.5, dtype)
    bias = draw(rng, (D, C), (1.0 / C) ** 0.5, dtype) if use_bias else None
    mw = draw(rng, (D, C), (1.0 / C) ** 0.5, dtype)
    mb = np.zeros((D,), dtype=np.float32)
    go = draw(rng, (B, D, T), 1.0, dtype)
    return x, w, bias, mw, mb, go


def kgen_inputs(meta, dtype: str, seed: int):
    """(logits [B, N*K, T], grad_kc [B, K, N, T]) for a kernel-generator case;
    meta = (B, N, K, T). Logits ~ N(0, 1.5^2), grad ~ N(0, 1)."""
    B, N, K, T = (int(v) for v in meta)
    rng = np.random.Generator(np.random.PCG64(seed))
    logits = draw(rng, (B, N * K, T), 1.5, dtype)
    gkc = draw(rng, (B, K, N, T), 1.0, dtype)
    return logits, gkc


def load_cases(path: str):
    """Yield dicts {name, meta, dtype, dist?, seed, <outputs>} from a golden .npz."""
    z = np.load(path, allow_pickle=False)
    names = sorted({k.split("/")[0] for k in z.files})
    for name in names:
        rec = {"name": name}
        for k in z.files:
            if k.startswith(name + "/"):
                v = z[k]
                rec[k.split("/", 1)[1]] = v.item() if v.ndim == 0 else v
        yield rec
