"""GPU parity of the fused dynamic conv (forward + backward) against the reference.

* golden: every fixture made from the reference's own formula, through the C ABI, for
  every plan that can run the shape (CUDA-core plan always, tcgen05 plan where legal);
* oracle: the hot shapes (D=256, K=3, N in {16..128}, dilations 1..32, offsets) against
  the float64 numpy oracle on identical inputs;
* autograd: the drop-in Python API (warmup -> cached plan consistency, backward);
* full size (B=16, T=4096): size-independent properties -- tcgen05 vs CUDA-core plan,
  exact linearity in grad_out (scaling by 2 is exact in floating point), determinism,
  and chunked-vs-whole equivalence.
"""

import os

import numpy as np
import pytest
import torch

from inputs import fdc_inputs, load_cases
from oracle import fdc_backward, fdc_forward
from parity import TORCH_DT, assert_close, to_dev

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "fdc_golden.npz")
CASES = list(load_cases(GOLDEN))


def _capi():
    from dudyconv_b200 import capi
    return capi


def run_capi(h, kc, mix, go, off, dil, plan):
    capi = _capi()
    out = torch.empty(h.shape[0], h.shape[1], kc.shape[3], device=h.device, dtype=h.dtype)
    capi.fdc_forward(h, kc, mix, out, off, dil, plan)
    gh = torch.full_like(h, float("nan"))  # every element must be written
    gk = torch.full_like(kc, float("nan"))
    gm = torch.full_like(mix, float("nan"))
    ws = torch.empty(max(256, capi.fdc_backward_workspace_size(h, kc, off, dil, plan)),
                     dtype=torch.uint8, device=h.device)
    capi.fdc_backward(go, h, kc, mix, gh, gk, gm, ws, off, dil, plan)
    torch.cuda.synchronize()
    assert capi.device_error() == 0
    return out, gh, gk, gm


def plans_for(h, kc, mix, off, dil):
    capi = _capi()
    B, D, L = h.shape
    _, K, N, T = kc.shape
    plans = [capi.PLAN_SIMT]
    if capi.lib().dudy_fdc_plan_available(capi.PLAN_TC, h.data_ptr(), kc.data_ptr(),
                                          mix.data_ptr(), B, D, L, T, N, K, off, dil,
                                          capi.dtype_code(h)):
        plans.append(capi.PLAN_TC)
    return plans


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_golden_capi(case):
    B, D, L, T, N, K, off, dil = (int(v) for v in case["meta"])
    dt = case["dtype"]
    h, kc, mix, go = fdc_inputs(case["meta"], dt, case["dist"], int(case["seed"]))
    th, tk, tm, tg = (to_dev(a, dt) for a in (h, kc, mix, go))
    for plan in plans_for(th, tk, tm, off, dil):
        out, gh, gk, gm = run_capi(th, tk, tm, tg, off, dil, plan)
        tag = f"{case['name']}/plan{plan}"
        assert_close(out, case["out"], dt, tag + "/out")
        assert_close(gh, case["grad_h"], dt, tag + "/grad_h")
        assert_close(gk, case["grad_kc"], dt, tag + "/grad_kc")
        assert_close(gm, case["grad_mix"], dt, tag + "/grad_mix")


def test_golden_hot_cases_use_tensor_cores():
    """The hot-path fixtures must be served by the tcgen05 plan, not a fallback."""
    capi = _capi()
    for case in CASES:
        if not case["name"].startswith("hot_") or case["dtype"] == "fp32":
            continue
        B, D, L, T, N, K, off, dil = (int(v) for v in case["meta"])
        h = torch.zeros(B, D, L, device="cuda", dtype=TORCH_DT[case["dtype"]])
        kc = torch.zeros(B, K, N, T, device="cuda", dtype=h.dtype)
        mix = torch.zeros(D, N, device="cuda", dtype=h.dtype)
        assert capi.fdc_default_plan(h, kc, mix, off, dil) == capi.PLAN_TC, case["name"]


def _draw(shape, std, dtype, gen):
    x = torch.randn(*shape, generator=gen, dtype=torch.float32) * std
    return x.to(TORCH_DT[dtype]).float().numpy()


HOT = [(N, dil, off, dt) for N in (16, 32, 64, 128) for dil, off in ((1, 0), (2, 64))
       for dt in ("fp16",)]
HOT += [(128, dil, 0, "fp16") for dil in (4, 8, 16, 32)]
HOT += [(128, 1, 0, "bf16"), (64, 3, 40, "bf16"), (128, 5, 96, "fp16")]


@pytest.mark.parametrize("N,dil,off,dt", HOT, ids=[f"N{a}_dil{b}_off{c}_{d}" for a, b, c, d in HOT])
def test_hot_shapes_vs_oracle(N, dil, off, dt):
    B, D, K, T = 2, 256, 3, 384
    L = off + T
    gen = torch.Generator().manual_seed(1000 + N + dil + off)
    h = _draw((B, D, L), 1.0, dt, gen)
    kc = _draw((B, K, N, T), (1.0 / N) ** 0.5, dt, gen)
    mix = _draw((D, N), (1.0 / 3) ** 0.5, dt, gen)
    go = _draw((B, D, T), 1.0, dt, gen)
    th, tk, tm, tg = (to_dev(a, dt) for a in (h, kc, mix, go))
    plans = plans_for(th, tk, tm, off, dil)
    assert _capi().PLAN_TC in plans
    out_ref = fdc_forward(h, kc, mix, off, dil)
    gh_ref, gk_ref, gm_ref = fdc_backward(go, h, kc, mix, off, dil)
    for plan in plans:
        out, gh, gk, gm = run_capi(th, tk, tm, tg, off, dil, plan)
        assert_close(out, out_ref, dt, f"plan{plan}/out")
        assert_close(gh, gh_ref, dt, f"plan{plan}/grad_h")
        assert_close(gk, gk_ref, dt, f"plan{plan}/grad_kc")
        assert_close(gm, gm_ref, dt, f"plan{plan}/grad_mix")


EDGE = [
    # (B, D, L, T, N, K, off, dil, dtype)  -- shapes outside the tensor-core envelope too
    (1, 1, 8, 8, 1, 1, 0, 1, "fp32"),
    (3, 128, 136, 136, 16, 1, 0, 1, "fp16"),     # K = 1
    (1, 128, 64, 8, 32, 4, 56, 7, "bf16"),       # T = 8 < tile, deep offset
    (2, 256, 300, 300, 64, 3, 0, 1, "fp16"),     # T % 8 != 0 -> CUDA-core plan
    (1, 192, 256, 256, 32, 3, 0, 1, "fp16"),     # D % 128 != 0 -> CUDA-core plan
    (1, 256, 512, 256, 128, 3, 256, 70, "fp16"), # halo beyond the tensor-core limit
    (1, 384, 256, 128, 64, 2, 64, 3, "bf16"),    # D = 3 halves (forward tc, backward simt)
    (2, 64, 520, 512, 24, 5, 8, 2, "fp32"),
    (2, 128, 272, 256, 128, 4, 16, 3, "bf16"),   # N = 128 with D = 128, K = 4
    (1, 256, 200, 200, 128, 3, 0, 1, "fp16"),    # N = 128, T not a multiple of the tile
    (3, 256, 1032, 1024, 128, 2, 8, 9, "fp16"),  # N = 128, K = 2, odd dilation, offset
    # 256-token chunks of a longer sequence (the model's call pattern): grad_h is zero
    # outside [off - (K-1)*dil, off + T), filled beside the grad_h kernel
    (2, 256, 1040, 256, 128, 3, 300, 8, "fp16"),  # 8-aligned taps, unaligned window start
    (2, 256, 1040, 256, 128, 3, 301, 1, "bf16"),  # shifted taps, unaligned window start
    (2, 128, 1040, 256, 64, 3, 782, 2, "fp16"),   # chunk ending 2 tokens before L
    # a single grad_kc work item (B = 1, K = 1, T <= 128): the backward grid has an idle CTA
    (1, 256, 64, 64, 128, 1, 0, 1, "fp16"),
    (1, 128, 96, 64, 16, 1, 32, 1, "bf16"),
]


@pytest.mark.parametrize("shape", EDGE, ids=[str(e) for e in EDGE])
def test_edge_shapes_vs_oracle(shape):
    B, D, L, T, N, K, off, dil, dt = shape
    gen = torch.Generator().manual_seed(7 + B + D + T)
    h = _draw((B, D, L), 0.5, dt, gen)
    kc = _draw((B, K, N, T), 0.5, dt, gen)
    mix = _draw((D, N), 0.5, dt, gen)
    go = _draw((B, D, T), 0.5, dt, gen)
    th, tk, tm, tg = (to_dev(a, dt) for a in (h, kc, mix, go))
    out_ref = fdc_forward(h, kc, mix, off, dil)
    gh_ref, gk_ref, gm_ref = fdc_backward(go, h, kc, mix, off, dil)
    out, gh, gk, gm = run_capi(th, tk, tm, tg, off, dil, _capi().PLAN_AUTO)
    assert_close(out, out_ref, dt, "out")
    assert_close(gh, gh_ref, dt, "grad_h")
    assert_close(gk, gk_ref, dt, "grad_kc")
    assert_close(gm, gm_ref, dt, "grad_mix")


def test_unaligned_view_falls_back_and_matches():
    """A contiguous view whose data pointer is not 16-byte aligned must still be right."""
    dt = "fp16"
    gen = torch.Generator().manual_seed(3)
    B, D, L, T, N, K = 1, 256, 128, 128, 32, 3
    base = torch.from_numpy(_draw((B * D * L + 1,), 1.0, dt, gen)).to("cuda", torch.float16)
    th = base[1:].view(B, D, L)
    kc = _draw((B, K, N, T), 0.2, dt, gen)
    mix = _draw((D, N), 0.5, dt, gen)
    go = _draw((B, D, T), 1.0, dt, gen)
    tk, tm, tg = (to_dev(a, dt) for a in (kc, mix, go))
    h = th.float().cpu().numpy()
    out, gh, gk, gm = run_capi(th, tk, tm, tg, 0, 1, _capi().PLAN_AUTO)
    assert_close(out, fdc_forward(h, kc, mix, 0, 1), dt, "out")
    ghr, gkr, gmr = fdc_backward(go, h, kc, mix, 0, 1)
    assert_close(gh, ghr, dt, "grad_h")
    assert_close(gk, gkr, dt, "grad_kc")
    assert_close(gm, gmr, dt, "grad_mix")


def test_autograd_api_and_plan_cache():
    import dudyconv_b200.cuda_ops as co
    dt = "fp16"
    gen = torch.Generator().manual_seed(11)
    B, D, L, T, N, K, off, dil = 2, 256, 640, 512, 64, 3, 128, 2
    h = _draw((B, D, L), 1.0, dt, gen)
    kc = _draw((B, K, N, T), 0.125, dt, gen)
    mix = _draw((D, N), 0.5, dt, gen)
    go = _draw((B, D, T), 1.0, dt, gen)
    th, tk, tm, tg = (to_dev(a, dt).requires_grad_(True) for a in (h, kc, mix, go))
    co.fused_dynamic_conv_forward_clear_warmup_cache()
    co.fused_dynamic_conv_backward_clear_warmup_cache()
    assert co.fused_dynamic_conv_forward_cached_plan_chunk(th, tk, tm, off, dil) == -1
    p = co.fused_dynamic_conv_forward_warmup_chunk(th, tk, tm, off, dil, repeat=1)
    assert p in (100, 200)
    assert co.fused_dynamic_conv_forward_cached_plan_chunk(th, tk, tm, off, dil) == p
    assert co.fused_dynamic_conv_forward_plan_name(p) in ("simt_generic", "tcgen05_tmem")
    pb = co.fused_dynamic_conv_backward_warmup_chunk(tg.detach(), th, tk, tm, off, dil, repeat=1)
    assert co.fused_dynamic_conv_backward_cached_plan_chunk(th, tk, off, dil) == pb
    out = co.fused_dynamic_conv_chunk(th, tk, tm, t_offset=off, dilation=dil)
    out.backward(tg.detach())
    assert_close(out, fdc_forward(h, kc, mix, off, dil), dt, "out")
    ghr, gkr, gmr = fdc_backward(go, h, kc, mix, off, dil)
    assert_close(th.grad, ghr, dt, "grad_h")
    assert_close(tk.grad, gkr, dt, "grad_kc")
    assert_close(tm.grad, gmr, dt, "grad_mix")
    # module wrapper with bias, whole-sequence form
    m = co.FusedDynamicConv1d(D, N, use_bias=True, dtype=torch.float16, device="cuda")
    y = m(th.detach()[:, :, :T].contiguous(), tk.detach(), dilation=1)
    assert y.shape == (B, D, T)


@pytest.fixture(scope="module")
def full_size():
    gen = torch.Generator(device="cuda").manual_seed(5)
    B, D, T, N, K = 16, 256, 4096, 128, 3
    h = torch.randn(B, D, T, device="cuda", generator=gen).half()
    kc = (torch.randn(B, K, N, T, device="cuda", generator=gen) * N ** -0.5).half()
    mix = (torch.randn(D, N, device="cuda", generator=gen) * 3 ** -0.5).half()
    go = torch.randn(B, D, T, device="cuda", generator=gen).half()
    return h, kc, mix, go


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def test_full_size_tc_matches_cuda_core_plan(full_size):
    h, kc, mix, go = full_size
    capi = _capi()
    assert capi.fdc_default_plan(h, kc, mix, 0, 1) == capi.PLAN_TC
    a = run_capi(h, kc, mix, go, 0, 1, capi.PLAN_TC)
    b = run_capi(h, kc, mix, go, 0, 1, capi.PLAN_SIMT)
    for x, y, name in zip(a, b, ("out", "grad_h", "grad_kc", "grad_mix")):
        assert torch.isfinite(x.float()).all(), name
        # both computed from identical fp16 inputs with fp32 accumulation
        assert _rel(x, y) < 2e-3, (name, _rel(x, y))


def test_full_size_linearity_and_determinism(full_size):
    h, kc, mix, go = full_size
    capi = _capi()
    a = run_capi(h, kc, mix, go, 0, 1, capi.PLAN_TC)
    a2 = run_capi(h, kc, mix, go, 0, 1, capi.PLAN_TC)
    s = run_capi(h, kc, mix, go * 2, 0, 1, capi.PLAN_TC)
    for x, y, z, name in zip(a, a2, s, ("out", "grad_h", "grad_kc", "grad_mix")):
        assert torch.equal(x, y), f"{name} not deterministic"
        if name == "grad_h":
            # doubling grad_out doubles every product and fp32 sum exactly; only results
            # whose fp16 rounding falls in the subnormal range (|v| < 2^-14) may differ
            normal = (x.float().abs() >= 2.0 ** -14) & (z.float().abs() >= 2.0 ** -13)
            assert torch.equal(z[normal], (x * 2)[normal]), f"{name} not exactly linear"
            assert float((z.float() - 2 * x.float()).abs().max()) <= 2.0 ** -23, name
        elif name != "out":
            # grad_kc / grad_mix contract the exact products G = go*h as G_hi + G_lo; only
            # G_lo terms in the fp16 subnormal range do not scale exactly
            assert _rel(z, x * 2) < 1e-5, (name, _rel(z, x * 2))


def test_full_size_chunked_equals_whole(full_size):
    """The model calls the op per 256-token chunk with t_offset; it must equal one call."""
    h, kc, mix, go = full_size
    capi = _capi()
    out_whole = run_capi(h, kc, mix, go, 0, 1, capi.PLAN_TC)[0]
    parts = []
    for s in range(0, 4096, 1024):
        kcs = kc[:, :, :, s:s + 1024].contiguous()
        o = torch.empty(16, 256, 1024, device="cuda", dtype=h.dtype)
        capi.fdc_forward(h, kcs, mix, o, s, 1, capi.PLAN_TC)
        parts.append(o)
    assert torch.equal(torch.cat(parts, dim=2), out_whole)
