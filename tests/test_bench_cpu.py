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


def test_clock_sampler_reads_nvml_reasons(monkeypatch):
    """The clock record reads SM clock, power and the clock-event reason bits; a fake NVML
    reports 1900 MHz under the power cap (bit 0x4) and nothing else."""
    import sys
    import time
    import types

    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=1, nvmlClocksEventReasonHwSlowdown=0x8,
        nvmlClocksEventReasonHwThermalSlowdown=0x40,
        nvmlClocksEventReasonSwThermalSlowdown=0x20, nvmlClocksEventReasonSwPowerCap=0x4,
        nvmlInit=lambda: None, nvmlShutdown=lambda: None,
        nvmlDeviceGetHandleByIndex=lambda i: ("gpu", i),
        nvmlDeviceGetMaxClockInfo=lambda h, c: 1965,
        nvmlDeviceGetClockInfo=lambda h, c: 1900,
        nvmlDeviceGetPowerUsage=lambda h: 812_000,
        nvmlDeviceGetCurrentClocksEventReasons=lambda h: 0x4 | 0x1)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    cs = bench.ClockSampler(3, period_s=0.002)
    cs.start()
    cs.wait_first_sample(5.0)
    time.sleep(0.05)
    cs.stop()
    r = cs.summary()
    assert r["source"] == "nvml" and r["samples"] >= 2
    assert r["sm_mhz"] == 1900.0 and r["sm_max_mhz"] == 1965.0 and r["power_w_max"] == 812.0
    assert r["reasons"] == ["sw_power_cap"]


def test_physical_gpu_follows_cuda_visible_devices(monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "5,2")
    assert bench.physical_gpu(0) == 5 and bench.physical_gpu(1) == 2
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert bench.physical_gpu(3) == 3


def test_physical_gpu_unknown_for_uuid_lists_without_nvml(monkeypatch):
    """A CUDA_VISIBLE_DEVICES of UUIDs (or a list shorter than the rank) gives no index, so
    the clock record is marked unsampled instead of reading another GPU's counters."""
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-1234abcd,GPU-5678ef00")
    assert bench.physical_gpu(0) is None
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3")
    assert bench.physical_gpu(1) is None
    s = bench.ClockSampler(None)
    s.start()
    s.stop()
    assert s.summary()["reasons"] == ["unsampled"]


def test_kernel_bounds_at_the_hot_shape():
    """On the measured peaks (6544 GB/s, 1601.5 TFLOP/s bf16) the forward and grad_h kernels
    are HBM-bound and the exact-product grad_kc/grad_mix kernel (51.5 GFLOP, 168 MB) is
    tensor-bound; at N = 64 the latter is HBM-bound."""
    alg = bench.algorithmic_bytes(16, 4096, 256, 128, 3)
    fl = bench.algorithmic_flops(16, 4096, 256, 128, 3)
    assert fl["fdc_tc_bk_n128_kernel"] == 4 * 2 * 16 * 4096 * 3 * 128 * 256
    bound = {k: bench.kernel_bound(alg[k], fl[k], 6544.3, 1601.5) for k in fl}
    assert bound["fdc_tc_conv_kernel<forward>"] == "hbm"
    assert bound["fdc_tc_conv2_kernel<grad_h>"] == "hbm"
    assert bound["fdc_tc_bk_n128_kernel"] == "tensor"
    alg64 = bench.algorithmic_bytes(16, 4096, 256, 64, 3)
    fl64 = bench.algorithmic_flops(16, 4096, 256, 64, 3)
    assert bench.kernel_bound(alg64["fdc_tc_bk_kernel"], fl64["fdc_tc_bk_kernel"], 6544.3,
                              1601.5) == "hbm"
    assert bench.kernel_bound(1000, None, 6544.3, 1601.5) == "hbm"
