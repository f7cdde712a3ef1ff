"""Full-size parity of the fused dynamic conv at the benchmark configurations.

Config 1: B=16, T=L=4096, D=256, K=3, N in {16, 32, 64, 128}, dilation 1, fp16 (and N=128
in bf16). Config 2: N=128 at dilations 2..32. Inputs follow the benchmark distributions
(h, go ~ N(0,1); kc ~ N(0,1/N); mix ~ N(0,1/3)).

Every output element is compared against the float64 restatement of the reference's
formula (``oracle/fdc_torch.py``, the same formula as ``oracle/fdc.py`` written in torch so
it runs on the GPU; pinned against the golden fixtures on the CPU). In particular the
grad_mix reduction over all 16 x 3 x 4096 terms and every CTA's partial, which only
happens at this size, is checked in full. Two sampled sequences are additionally checked
against the numpy oracle itself. Tolerance: the fixed fp16/bf16 bar of ``tests/parity.py``
(|got - ref| <= 2e-3 + 1e-2 |ref|).
"""

import numpy as np
import pytest
import torch

from oracle import fdc_backward, fdc_forward
from oracle.fdc_torch import fdc_backward_t, fdc_forward_t
from parity import assert_close, assert_close_t

pytestmark = pytest.mark.gpu

CFG = [(N, 1, "fp16") for N in (16, 32, 64, 128)]
CFG += [(128, d, "fp16") for d in (2, 4, 8, 16, 32)]
CFG += [(128, 1, "bf16")]

B, D, T, K = 16, 256, 4096, 3


def _inputs(N, dt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    tdt = torch.float16 if dt == "fp16" else torch.bfloat16
    h = torch.randn(B, D, T, device="cuda", generator=g).to(tdt)
    kc = (torch.randn(B, K, N, T, device="cuda", generator=g) * N ** -0.5).to(tdt)
    mix = (torch.randn(D, N, device="cuda", generator=g) * 3 ** -0.5).to(tdt)
    go = torch.randn(B, D, T, device="cuda", generator=g).to(tdt)
    return h, kc, mix, go


def _run(h, kc, mix, go, dil):
    from dudyconv_b200 import capi
    assert capi.fdc_default_plan(h, kc, mix, 0, dil) == capi.PLAN_TC
    out = torch.empty(B, D, T, device="cuda", dtype=h.dtype)
    capi.fdc_forward(h, kc, mix, out, 0, dil)
    gh = torch.full_like(h, float("nan"))
    gk = torch.full_like(kc, float("nan"))
    gm = torch.full_like(mix, float("nan"))
    ws = torch.empty(capi.fdc_backward_workspace_size(h, kc, 0, dil), dtype=torch.uint8,
                     device="cuda")
    capi.fdc_backward(go, h, kc, mix, gh, gk, gm, ws, 0, dil)
    torch.cuda.synchronize()
    assert capi.device_error() == 0
    return out, gh, gk, gm


@pytest.mark.parametrize("N,dil,dt", CFG, ids=[f"N{n}_dil{d}_{t}" for n, d, t in CFG])
def test_full_size_vs_oracle(N, dil, dt):
    h, kc, mix, go = _inputs(N, dt, 7000 + N + dil)
    out, gh, gk, gm = _run(h, kc, mix, go, dil)
    # every element against the float64 formula, on the device
    assert_close_t(out, fdc_forward_t(h, kc, mix, 0, dil), dt, "out")
    rgh, rgk, rgm = fdc_backward_t(go, h, kc, mix, 0, dil)
    assert_close_t(gh, rgh, dt, "grad_h")
    del rgh
    assert_close_t(gk, rgk, dt, "grad_kc")
    del rgk
    assert_close_t(gm, rgm, dt, "grad_mix")
    # two sampled sequences against the numpy oracle (outputs of one sequence depend only
    # on that sequence)
    for b in (3, 14):
        hn, kn, gn = (x[b:b + 1].float().cpu().numpy() for x in (h, kc, go))
        mn = mix.float().cpu().numpy()
        assert_close(out[b:b + 1], fdc_forward(hn, kn, mn, 0, dil), dt, f"seq{b}/out")
        rgh1, rgk1, _ = fdc_backward(gn, hn, kn, mn, 0, dil)
        assert_close(gh[b:b + 1], rgh1, dt, f"seq{b}/grad_h")
        assert_close(gk[b:b + 1], rgk1, dt, f"seq{b}/grad_kc")


def test_torch_oracle_matches_numpy_oracle_on_gpu():
    """The device-side float64 restatement equals the numpy oracle (small shape, on the
    GPU this time, so the full-size checks above rest on a pinned checker)."""
    g = torch.Generator().manual_seed(3)
    Bs, Ds, Ls, Ts, Ns, Ks, off, dil = 2, 64, 200, 160, 16, 3, 40, 3
    h = torch.randn(Bs, Ds, Ls, generator=g, dtype=torch.float64)
    kc = torch.randn(Bs, Ks, Ns, Ts, generator=g, dtype=torch.float64)
    mix = torch.randn(Ds, Ns, generator=g, dtype=torch.float64)
    go = torch.randn(Bs, Ds, Ts, generator=g, dtype=torch.float64)
    got = [fdc_forward_t(*(x.cuda() for x in (h, kc, mix)), off, dil)]
    got += list(fdc_backward_t(*(x.cuda() for x in (go, h, kc, mix)), off, dil))
    want = [fdc_forward(h.numpy(), kc.numpy(), mix.numpy(), off, dil)]
    want += list(fdc_backward(go.numpy(), h.numpy(), kc.numpy(), mix.numpy(), off, dil))
    for a, b_ in zip(got, want):
        np.testing.assert_allclose(a.cpu().numpy(), b_, rtol=1e-12, atol=1e-12)
