"""Pin the numpy oracle against the reference's own formulas (golden fixtures).

The fixtures were produced by ``tests/golden/make_golden.py``, which imports the
reference's ``torch_reference_materialized_chunk`` and
``torch_reference_source_conv_mixed_chunk`` and differentiates them in float64.
"""

import os

import numpy as np
import pytest

from inputs import fdc_inputs, fscm_inputs, load_cases, round_to
from oracle import fdc_backward, fdc_forward, fscm_backward, fscm_forward

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
FDC = list(load_cases(os.path.join(GOLDEN, "fdc_golden.npz")))
FSCM = list(load_cases(os.path.join(GOLDEN, "fscm_golden.npz")))


def _close(a, b, name):
    # golden outputs are float32 roundings of float64 values
    scale = max(1e-30, float(np.abs(b).max()))
    np.testing.assert_allclose(a, b, rtol=2e-6, atol=2e-6 * scale, err_msg=name)


@pytest.mark.parametrize("case", FDC, ids=[c["name"] for c in FDC])
def test_fdc_oracle_matches_reference(case):
    meta = case["meta"]
    B, D, L, T, N, K, off, dil = (int(v) for v in meta)
    h, kc, mix, go = fdc_inputs(meta, case["dtype"], case["dist"], int(case["seed"]))
    out = fdc_forward(h, kc, mix, off, dil)
    gh, gk, gm = fdc_backward(go, h, kc, mix, off, dil)
    _close(out, case["out"], "out")
    _close(gh, case["grad_h"], "grad_h")
    _close(gk, case["grad_kc"], "grad_kc")
    _close(gm, case["grad_mix"], "grad_mix")
    # grad_h is zero outside [off-(K-1)*dil, off+T)
    lo = max(0, off - (K - 1) * dil)
    assert not gh[:, :, :lo].any() and not gh[:, :, off + T:].any()


@pytest.mark.parametrize("case", FSCM, ids=[c["name"] for c in FSCM])
def test_fscm_oracle_matches_reference(case):
    meta = case["meta"]
    B, D, L, T, C, S, off, dil, use_bias = (int(v) for v in meta)
    x, w, bias, mw, mb, go = fscm_inputs(meta, case["dtype"], int(case["seed"]))
    out = fscm_forward(x, w, bias, mw, mb, off, T, dil)
    gx, gw, gb, gmw, gmb = fscm_backward(go, x, w, bias, mw, mb, off, T, dil)
    _close(out, case["out"], "out")
    _close(gx, case["grad_x"], "grad_x")
    _close(gw, case["grad_w"], "grad_w")
    _close(gmw, case["grad_mix_w"], "grad_mix_w")
    _close(gmb, case["grad_mix_b"], "grad_mix_b")
    if use_bias:
        _close(gb, case["grad_bias"], "grad_bias")
    else:
        assert gb is None


def test_oracle_detects_planted_error():
    """The checker must fail on a wrong answer: plant an off-by-one tap shift."""
    case = next(c for c in FDC if c["name"] == "odd_dilation2")
    meta = case["meta"]
    B, D, L, T, N, K, off, dil = (int(v) for v in meta)
    h, kc, mix, go = fdc_inputs(meta, case["dtype"], case["dist"], int(case["seed"]))
    wrong = fdc_forward(h, kc, mix, off, dil + 1)
    with pytest.raises(AssertionError):
        _close(wrong, case["out"], "out")


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.1415927, 65504.0, 1e-40], dtype=np.float32)
    r = round_to(x, "bf16")
    # 1 + 2^-8 is a tie between 1.0 and 1.0078125 -> even (1.0)
    assert r[0] == 1.0 and r[1] == 1.0
    assert r[2] == np.float32(1.015625)
    assert (r.view(np.uint32) & 0xFFFF).max() == 0


@pytest.mark.parametrize("case", FDC, ids=[c["name"] for c in FDC])
def test_fdc_torch_oracle_matches_reference(case):
    """The torch float64 restatement (used for the full-size GPU checks) equals the
    reference's formulas on every golden case."""
    import torch

    from oracle.fdc_torch import fdc_backward_t, fdc_forward_t

    meta = case["meta"]
    B, D, L, T, N, K, off, dil = (int(v) for v in meta)
    h, kc, mix, go = (torch.from_numpy(np.ascontiguousarray(a, dtype=np.float64))
                      for a in fdc_inputs(meta, case["dtype"], case["dist"], int(case["seed"])))
    out = fdc_forward_t(h, kc, mix, off, dil)
    gh, gk, gm = fdc_backward_t(go, h, kc, mix, off, dil)
    _close(out.numpy(), case["out"], "out")
    _close(gh.numpy(), case["grad_h"], "grad_h")
    _close(gk.numpy(), case["grad_kc"], "grad_kc")
    _close(gm.numpy(), case["grad_mix"], "grad_mix")


KGEN = list(load_cases(os.path.join(GOLDEN, "kgen_golden.npz")))


@pytest.mark.parametrize("case", KGEN, ids=[c["name"] for c in KGEN])
def test_kernel_gen_oracle_matches_reference(case):
    """The numpy restatement of the kernel generator's tail equals the reference model's
    own _logits_to_kernel and its autograd backward."""
    from inputs import kgen_inputs
    from oracle.kernel_gen import logits_to_kernel, logits_to_kernel_backward

    B, N, K, T = (int(v) for v in case["meta"])
    logits, gkc = kgen_inputs(case["meta"], case["dtype"], int(case["seed"]))
    _close(logits_to_kernel(logits, N, K), case["kc"], "kc")
    _close(logits_to_kernel_backward(logits, gkc, N, K), case["grad_logits"], "grad_logits")
