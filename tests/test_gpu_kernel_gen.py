"""GPU parity of the fused kernel-generator tail (softmax over K + flip + layout change).

``dudy_logits_to_kernel`` / ``dudy_logits_to_kernel_backward`` against the golden fixtures
made from the reference model's own ``_logits_to_kernel``
(``backbone_dil_unshared.py:1821-1900``) and against the numpy oracle at the model's shape
(N=128, K=3) and at shapes that take the other code paths (K outside the unrolled set,
T not a multiple of 8, an unaligned view); then the composed
``fused_dynamic_conv_chunk_from_logits`` forward + backward against the oracle chain.
Tolerances: the fixed bar of tests/parity.py.
"""

import os

import numpy as np
import pytest
import torch

from inputs import fdc_inputs, kgen_inputs, load_cases
from oracle import fdc_backward, fdc_forward
from oracle.kernel_gen import logits_to_kernel, logits_to_kernel_backward
from parity import TORCH_DT, assert_close, to_dev

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kgen_golden.npz")
CASES = list(load_cases(GOLDEN))


def _run(tl, tg, N, K):
    from dudyconv_b200 import capi
    B, _, T = tl.shape
    kc = torch.full((B, K, N, T), float("nan"), device="cuda", dtype=tl.dtype)
    capi.logits_to_kernel(tl, kc)
    gl = torch.full_like(tl, float("nan"))
    capi.logits_to_kernel_backward(kc, tg, gl)
    torch.cuda.synchronize()
    return kc, gl


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_golden(case):
    B, N, K, T = (int(v) for v in case["meta"])
    dt = case["dtype"]
    logits, gkc = kgen_inputs(case["meta"], dt, int(case["seed"]))
    kc, gl = _run(to_dev(logits, dt), to_dev(gkc, dt), N, K)
    assert_close(kc, case["kc"], dt, "kc")
    # the backward reads the rounded kc (the forward's output), as autograd would
    kcr = kc.float().cpu().numpy().astype(np.float64)
    dot = (kcr * gkc).sum(axis=1, keepdims=True)
    want = np.ascontiguousarray((kcr * (gkc - dot))[:, ::-1].transpose(0, 2, 1, 3)
                                .reshape(B, N * K, T))
    assert_close(gl, want, dt, "grad_logits")
    if dt == "fp32":
        assert_close(gl, case["grad_logits"], dt, "grad_logits vs reference")


SHAPES = [(16, 128, 3, 4096, "fp16"), (2, 128, 3, 256, "bf16"), (2, 16, 7, 96, "fp16"),
          (1, 32, 12, 64, "fp32"), (3, 8, 3, 37, "fp16"), (1, 4, 2, 8, "bf16")]


@pytest.mark.parametrize("B,N,K,T,dt", SHAPES, ids=[f"B{b}_N{n}_K{k}_T{t}_{d}"
                                                     for b, n, k, t, d in SHAPES])
def test_vs_oracle(B, N, K, T, dt):
    logits, gkc = kgen_inputs([B, N, K, T], dt, 99 + N + K + T)
    kc, gl = _run(to_dev(logits, dt), to_dev(gkc, dt), N, K)
    assert_close(kc, logits_to_kernel(logits, N, K), dt, "kc")
    # the softmax backward works from the forward's rounded output, as autograd does in
    # the reference (PyTorch's softmax backward reads the saved 16-bit output)
    kcr = kc.double().cpu().numpy()
    dot = (kcr * gkc).sum(axis=1, keepdims=True)
    want = np.ascontiguousarray((kcr * (gkc - dot))[:, ::-1].transpose(0, 2, 1, 3)
                                .reshape(B, N * K, T))
    assert_close(gl, want, dt, "grad_logits")
    if dt != "bf16":
        # for fp16 / fp32 the rounding of kc also stays within the bar of the exact chain
        assert_close(gl, logits_to_kernel_backward(logits, gkc, N, K), dt, "grad_logits exact")


def test_unaligned_view_and_autograd_function():
    from dudyconv_b200.kernel_gen import logits_to_kernel as fused

    B, N, K, T = 2, 16, 3, 64
    logits, gkc = kgen_inputs([B, N, K, T], "fp16", 5)
    base = torch.empty(B * N * K * T + 1, device="cuda", dtype=torch.float16)
    tl = base[1:].view(B, N * K, T)
    tl.copy_(to_dev(logits, "fp16"))
    tl.requires_grad_(True)
    kc = fused(tl, N, K)
    kc.backward(to_dev(gkc, "fp16"))
    assert_close(kc, logits_to_kernel(logits, N, K), "fp16", "kc")
    assert_close(tl.grad, logits_to_kernel_backward(logits, gkc, N, K), "fp16", "grad_logits")


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_op_from_logits(dt):
    """fused_dynamic_conv_chunk_from_logits = the op applied to _logits_to_kernel(logits),
    forward and backward (grad_logits through the op's 16-bit grad_kc, as the reference's
    chain of autograd steps computes it)."""
    from dudyconv_b200 import capi
    from dudyconv_b200.kernel_gen import fused_dynamic_conv_chunk_from_logits

    B, D, L, T, N, K, off, dil = 2, 256, 384, 256, 128, 3, 128, 1
    h, _, mix, go = fdc_inputs([B, D, L, T, N, K, off, dil], dt, "base", 31)
    logits, _ = kgen_inputs([B, N, K, T], dt, 32)
    th, tm, tl = (to_dev(a, dt).requires_grad_(True) for a in (h, mix, logits))
    tg = to_dev(go, dt)
    out = fused_dynamic_conv_chunk_from_logits(th, tl, tm, t_offset=off, dilation=dil)
    out.backward(tg)
    # the same steps one by one through the C ABI
    kc_dev = torch.empty(B, K, N, T, device="cuda", dtype=TORCH_DT[dt])
    capi.logits_to_kernel(tl.detach(), kc_dev)
    gh_d, gk_d, gm_d = (torch.empty_like(x) for x in (th, kc_dev, tm))
    ws = torch.empty(capi.fdc_backward_workspace_size(th, kc_dev, off, dil), device="cuda",
                     dtype=torch.uint8)
    capi.fdc_backward(tg, th.detach(), kc_dev, tm.detach(), gh_d, gk_d, gm_d, ws, off, dil)
    torch.cuda.synchronize()
    kc16 = kc_dev.double().cpu().numpy()
    assert_close(kc_dev, logits_to_kernel(logits, N, K), dt, "kc")
    assert_close(out, fdc_forward(h, kc16, mix, off, dil), dt, "out")
    gh, _, gm = fdc_backward(go, h, kc16, mix, off, dil)
    assert_close(th.grad, gh, dt, "grad_h")
    assert_close(tm.grad, gm, dt, "grad_mix")
    gk16 = gk_d.double().cpu().numpy()
    dot = (kc16 * gk16).sum(axis=1, keepdims=True)
    want = np.ascontiguousarray((kc16 * (gk16 - dot))[:, ::-1].transpose(0, 2, 1, 3)
                                .reshape(B, N * K, T))
    assert_close(tl.grad, want, dt, "grad_logits")
