"""The byte counts behind bench.py's roofline fractions: the whole fwd+bwd step and the
per-kernel algorithmic bytes at the hot shape (B=16, T=4096, D=256, K=3, fp16)."""

import bench


def test_step_bytes_match_the_op_minimum_traffic():
    # forward: read h, kc, mix, write out; backward: read go, h, kc, mix, write grad_h,
    # grad_kc, grad_mix (2 bytes per element)
    expected = {16: 186.7e6, 32: 205.6e6, 64: 243.4e6, 128: 319.0e6}
    for N, mb in expected.items():
        r = bench.step_roofline(16, 4096, 256, N, 3, 1.0, 6500.0, "measured")
        assert abs(r["algorithmic_bytes_per_step"] - mb) < 0.05e6, (N, r)


def test_step_roofline_fraction():
    r = bench.step_roofline(16, 4096, 256, 128, 3, 0.112, 6461.2, "measured")
    assert abs(r["achieved"] - 318963712 / 0.112e-3 / 1e9) < 1e-6
    assert abs(r["frac"] - r["achieved"] / 6461.2) < 1e-12
    assert r["bound"] == "hbm" and r["unit"] == "GB/s"


def test_kernel_bytes_at_the_hot_shape():
    alg = bench.algorithmic_bytes(16, 4096, 256, 128, 3)
    assert alg["fdc_tc_conv_kernel<forward>"] == 117506048
    assert alg["fdc_tc_conv2_kernel<grad_h>"] == 117506048
    assert alg["fdc_tc_bk_n128_kernel"] == 167903232
    # the three kernels together read/write the step's bytes plus go/kc/mix twice
    step = bench.step_roofline(16, 4096, 256, 128, 3, 1.0, 1.0, "x")["algorithmic_bytes_per_step"]
    assert sum(alg[k] for k in ("fdc_tc_conv_kernel<forward>", "fdc_tc_conv2_kernel<grad_h>",
                                "fdc_tc_bk_n128_kernel")) > step
