"""Failure detection on the GPU without a fault: a bounded wait that runs out.

Every mbarrier wait in the tensor-core kernels is bounded; on expiry the wait records its
site in the device error record, raises the CTA's abort flag (so the CTA's other roles
stop waiting too), and the CTA frees its TMEM and returns instead of hanging. Here a
self-test kernel built like those kernels waits, with a 2 ms limit, on an mbarrier that
nothing arrives at. The test checks that the kernel returns, that both warps report the
give-up (one by its own timeout, one through the abort flag), that
``dudy_device_error_info`` names the wait site, block, thread and counter, that the
record can be cleared, and that the same context then still computes correct results.
No GPU fault, trap or hang is involved.
"""

import time

import numpy as np
import pytest
import torch

from oracle import fdc_backward, fdc_forward
from parity import assert_close, to_dev

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports_its_site():
    from dudyconv_b200 import capi

    capi.device_error(reset=True)
    assert capi.device_error_info() == (0, 0, 0, 0)
    t0 = time.time()
    assert capi.selftest_wait_timeout(2000) == (0, 0)
    assert time.time() - t0 < 5.0
    site, block, thread, counter = capi.device_error_info(reset=True)
    assert (site, block, thread, counter) == (901, 0, 0, 7)
    assert capi.device_error_info() == (0, 0, 0, 0)

    # the context is still usable: a tensor-core forward + backward afterwards is correct
    gen = np.random.Generator(np.random.PCG64(11))
    B, D, L, T, N, K, off, dil = 1, 256, 256, 256, 128, 3, 0, 1
    h = gen.standard_normal((B, D, L), dtype=np.float32)
    kc = gen.standard_normal((B, K, N, T), dtype=np.float32) * N ** -0.5
    mix = gen.standard_normal((D, N), dtype=np.float32) * 3 ** -0.5
    go = gen.standard_normal((B, D, T), dtype=np.float32)
    h, kc, mix, go = (a.astype(np.float16).astype(np.float32) for a in (h, kc, mix, go))
    th, tk, tm, tg = (to_dev(a, "fp16") for a in (h, kc, mix, go))
    assert capi.fdc_default_plan(th, tk, tm, off, dil) == capi.PLAN_TC
    out = torch.empty(B, D, T, device="cuda", dtype=torch.float16)
    capi.fdc_forward(th, tk, tm, out, off, dil)
    gh, gk, gm = torch.empty_like(th), torch.empty_like(tk), torch.empty_like(tm)
    ws = torch.empty(capi.fdc_backward_workspace_size(th, tk, off, dil), dtype=torch.uint8,
                     device="cuda")
    capi.fdc_backward(tg, th, tk, tm, gh, gk, gm, ws, off, dil)
    torch.cuda.synchronize()
    assert capi.device_error() == 0
    assert_close(out, fdc_forward(h, kc, mix, off, dil), "fp16", "out")
    for got, want, name in zip((gh, gk, gm), fdc_backward(go, h, kc, mix, off, dil),
                               ("grad_h", "grad_kc", "grad_mix")):
        assert_close(got, want, "fp16", name)


def test_selftest_rejects_bad_limits():
    from dudyconv_b200 import capi

    for bad in (0, -5, 2_000_000):
        with pytest.raises(capi.DudyError):
            capi.selftest_wait_timeout(bad)
