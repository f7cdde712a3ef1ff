"""The allocation-free backward entry point, for callers that cannot allocate device
memory at call time (a process whose device memory is fixed at start-up, code where
cudaMalloc is not allowed or would synchronize the device, or a foreign-function caller
with no allocator to pass a workspace from).

dudy_fdc_backward_noalloc keeps its scratch in a fixed array inside the library instead
of a caller workspace. It runs the same deterministic kernels as the workspace entry
point dudy_fdc_backward, so through the C ABI its results must be bitwise equal to that
entry point's, on the tensor-core plan and on the CUDA-core plan, including for calls
queued back to back on one stream with different inputs and no synchronisation in
between (the second call's partial sums reuse the array right after the first call's
reduction reads it). Shapes that need more scratch than the fixed array are refused
before any work is enqueued. This file is collected last so a run that stops at the
first failure has run every other test before it.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(B, D, L, T, N, K, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    h = torch.randn(B, D, L, device="cuda", generator=g).to(dtype)
    kc = (torch.randn(B, K, N, T, device="cuda", generator=g) * N ** -0.5).to(dtype)
    mix = (torch.randn(D, N, device="cuda", generator=g) * 3 ** -0.5).to(dtype)
    go = torch.randn(B, D, T, device="cuda", generator=g).to(dtype)
    return h, kc, mix, go


CASES = [
    # (B, D, L, T, N, K, off, dil, dtype, tag, expected plan)
    (2, 256, 512, 512, 128, 3, 0, 1, torch.float16, "fp16", 200),   # tcgen05 plan
    (1, 256, 640, 384, 64, 3, 256, 2, torch.bfloat16, "bf16", 200),  # chunk offset, shifted taps
    (2, 96, 200, 168, 24, 4, 32, 3, torch.float32, "fp32", 100),     # CUDA-core plan
]


@pytest.mark.parametrize("case", CASES, ids=[c[9] + f"_D{c[1]}" for c in CASES])
def test_noalloc_matches_workspace_backward_twice(case):
    from dudyconv_b200 import capi

    B, D, L, T, N, K, off, dil, dtype, tag, want_plan = case
    sets = [_inputs(B, D, L, T, N, K, dtype, seed=B + D + T + 17 * i) for i in range(2)]
    assert capi.fdc_default_plan(*sets[0][:3], off, dil) == want_plan
    # the existing entry point, with a caller workspace, one input set at a time
    refs = []
    for h, kc, mix, go in sets:
        ref = [torch.empty_like(h), torch.empty_like(kc), torch.empty_like(mix)]
        ws = torch.empty(max(256, capi.fdc_backward_workspace_size(h, kc, off, dil)),
                         dtype=torch.uint8, device="cuda")
        capi.fdc_backward(go, h, kc, mix, *ref, ws, off, dil)
        torch.cuda.synchronize()
        refs.append(ref)
    for rnd in range(2):
        # two calls queued back to back on the current stream, no synchronisation between
        gots = []
        for h, kc, mix, go in sets:
            got = [torch.full_like(h, float("nan")), torch.full_like(kc, float("nan")),
                   torch.full_like(mix, float("nan"))]
            capi.fdc_backward_noalloc(go, h, kc, mix, *got, off, dil)
            gots.append(got)
        torch.cuda.synchronize()
        assert capi.device_error() == 0
        for i, (got, ref) in enumerate(zip(gots, refs)):
            for name, g, r in zip(("grad_h", "grad_kc", "grad_mix"), got, ref):
                assert torch.equal(g, r), f"round {rnd}, input set {i}: {name} differs"


def test_noalloc_refuses_oversized_scratch():
    from dudyconv_b200 import capi

    lib = capi.lib()
    # D=8192, N=1024 needs a D*N fp32 partial of 32 MiB, above the fixed 20 MiB array
    B, D, L, T, N, K = 1, 8192, 8, 8, 1024, 1
    h = torch.zeros(B, D, L, device="cuda", dtype=torch.float16)
    kc = torch.zeros(B, K, N, T, device="cuda", dtype=torch.float16)
    mix = torch.zeros(D, N, device="cuda", dtype=torch.float16)
    go = torch.zeros(B, D, T, device="cuda", dtype=torch.float16)
    gh = torch.full_like(h, 7.0)
    gk = torch.full_like(kc, 7.0)
    gm = torch.full_like(mix, 7.0)
    need = capi.fdc_backward_workspace_size(h, kc, 0, 1)
    assert need > 20 * 1024 * 1024
    rc = lib.dudy_fdc_backward_noalloc(h.data_ptr(), h.data_ptr(), kc.data_ptr(), mix.data_ptr(),
                                       gh.data_ptr(), gk.data_ptr(), gm.data_ptr(), B, D, L, T, N,
                                       K, 0, 1, capi.DTYPE_F16, capi.PLAN_AUTO,
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rc == capi.ERR_WORKSPACE
    assert "more than the fixed" in capi.last_error()
    assert bool((gh == 7).all()) and bool((gk == 7).all()) and bool((gm == 7).all())
