"""Shared helpers of the GPU parity tests.

Tolerances (stated once, used everywhere; the project's parity bar):
  * fp32 inputs : rtol = 1e-5, atol = 1e-5 * max|ref|   (elementwise relative error is
                  undefined at exact zeros, so atol is tied to the tensor's scale)
  * fp16 / bf16 : rtol = 1e-2, atol = 2e-3, both fixed, on outputs and every gradient:
                  |got - ref| <= 2e-3 + 1e-2 * |ref| elementwise.
The reference side is always the float64 oracle (or the golden fixture made from the
reference's own formulas) evaluated on the exact same (16-bit rounded) inputs.
"""

from __future__ import annotations

import numpy as np
import torch

TORCH_DT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def tol(dtype: str, ref: np.ndarray):
    scale = float(np.abs(ref).max()) if ref.size else 0.0
    if dtype == "fp32":
        return 1e-5, 1e-5 * max(scale, 1e-30)
    return 1e-2, 2e-3


def assert_close(actual: torch.Tensor, ref: np.ndarray, dtype: str, name: str):
    a = actual.detach().float().cpu().numpy().astype(np.float64)
    r = np.asarray(ref, dtype=np.float64)
    assert a.shape == r.shape, (name, a.shape, r.shape)
    rtol, atol = tol(dtype, r)
    err = np.abs(a - r)
    bound = atol + rtol * np.abs(r)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(
            f"{name} [{dtype}]: {int(bad.sum())}/{err.size} elements out of tolerance "
            f"(rtol={rtol:g}, atol={atol:g}); worst at {i}: got {a[i]!r}, want {r[i]!r}; "
            f"max abs err {float(err.max()):.3e}")


def to_dev(x: np.ndarray, dtype: str, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).to(device=device, dtype=TORCH_DT[dtype])


def assert_close_t(actual: torch.Tensor, ref: torch.Tensor, dtype: str, name: str):
    """assert_close with both sides as tensors on one device (full-size checks, where a
    copy to numpy would dominate); ``ref`` is float64."""
    a = actual.detach().double()
    r = ref.detach().double()
    assert a.shape == r.shape, (name, tuple(a.shape), tuple(r.shape))
    scale = float(r.abs().max()) if r.numel() else 0.0
    if dtype == "fp32":
        rtol, atol = 1e-5, 1e-5 * max(scale, 1e-30)
    else:
        rtol, atol = 1e-2, 2e-3
    err = (a - r).abs()
    bound = atol + rtol * r.abs()
    bad = err > bound
    nbad = int(bad.sum())
    if nbad:
        i = int(torch.argmax((err - bound).flatten()))
        idx = np.unravel_index(i, tuple(a.shape))
        raise AssertionError(
            f"{name} [{dtype}]: {nbad}/{err.numel()} elements out of tolerance "
            f"(rtol={rtol:g}, atol={atol:g}); worst at {idx}: got "
            f"{float(a.flatten()[i])!r}, want {float(r.flatten()[i])!r}; "
            f"max abs err {float(err.max()):.3e}")
