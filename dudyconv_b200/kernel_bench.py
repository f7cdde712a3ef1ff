"""Per-kernel timing of the fused dynamic conv through the C ABI.

    python -m dudyconv_b200.kernel_bench [--batch 16 --seq 4096 --basis 128 --dilation 1]
           [--stage all|forward|grad_h|grad_kc_mix] [--plan tc|simt] [--iters 50]
           [--profile]
    python -m dudyconv_b200.kernel_bench --op fscm [--channels 16 --taps 3 --dilation 1]


Times each stage (forward, grad_h, grad_kc + grad_mix) with CUDA events, rotating two
input sets so every launch streams from HBM, and prints one JSON line. ``--profile``
runs three warm-up launches of the chosen stage and then exactly one more, for an
``ncu -k <kernel> -s 3 -c 1`` capture of that launch.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import capi

STAGES = ("forward", "grad_h", "grad_kc_mix")


def algorithmic_bytes(stage, B, T, D, N, K, es=2):
    bt = B * T
    if stage in ("forward", "grad_h"):
        return (2 * bt * D + bt * K * N + D * N) * es
    return (2 * bt * D + 2 * bt * K * N + 2 * D * N) * es


def fscm_main(a):
    """Source conv (fused_source_conv_mixed) forward and backward through the C ABI.
    Algorithmic bytes: forward x + out, backward go + x + grad_x (parameters are KB)."""
    dev = torch.device("cuda")
    dt = torch.float16 if a.dtype == "fp16" else torch.bfloat16
    B, T, D, C, S, dil = a.batch, a.seq, a.dim, a.channels, a.taps, a.dilation
    L = T
    gen = torch.Generator(device=dev).manual_seed(0)

    def make():
        return (torch.randn(B, D, L, device=dev, generator=gen).to(dt),
                (torch.randn(D, C, S, device=dev, generator=gen) * 3 ** -0.5).to(dt),
                (torch.randn(D, C, device=dev, generator=gen) * C ** -0.5).to(dt),
                (torch.randn(D, C, device=dev, generator=gen) * C ** -0.5).to(dt),
                torch.zeros(D, device=dev, dtype=dt),
                torch.randn(B, D, T, device=dev, generator=gen).to(dt))

    sets = [make() for _ in range(2)]
    out = torch.empty(B, D, T, device=dev, dtype=dt)
    x0, w0 = sets[0][0], sets[0][1]
    gx = torch.empty_like(x0)
    gw = torch.empty_like(w0)
    gb = torch.empty(D, C, device=dev, dtype=dt)
    gmw = torch.empty(D, C, device=dev, dtype=dt)
    gmb = torch.empty(D, device=dev, dtype=dt)
    ws = torch.empty(max(256, capi.fscm_backward_workspace_size(x0, w0, 0, T, dil)),
                     dtype=torch.uint8, device=dev)

    def launch(stage, i):
        x, w, bias, mw, mb, go = sets[i % 2]
        if stage == "forward":
            capi.fscm_forward(x, w, bias, mw, mb, out, 0, T, dil)
        else:
            capi.fscm_backward(go, x, w, bias, mw, mb, gx, gw, gb, gmw, gmb, ws, 0, T, dil)

    if a.profile:  # 4 launches of each pass, nothing timed (for ncu -k ... -s 3 -c 1)
        for st in ("forward", "backward"):
            for i in range(4):
                launch(st, i)
        torch.cuda.synchronize()
        print(json.dumps({"profile_launches": 4, "device_error": capi.device_error_info()}))
        return
    bt = B * T
    alg = {"forward": 2 * bt * D * 2, "backward": 3 * bt * D * 2}
    res = {"op": "fscm", "batch": B, "seq": T, "D": D, "C": C, "S": S, "dilation": dil,
           "dtype": a.dtype, "gelu_per_forward": bt * D * C}
    for st in ("forward", "backward"):
        for i in range(3):
            launch(st, i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(a.iters):
            launch(st, i)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / a.iters * 1e3
        res[st] = {"us": us, "GB/s": alg[st] / us / 1e3}
    res["device_error"] = capi.device_error_info()
    print(json.dumps(res))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="fdc", choices=["fdc", "fscm"])
    ap.add_argument("--channels", type=int, default=16, help="fscm: source channels C")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--basis", type=int, default=128)
    ap.add_argument("--taps", type=int, default=3)
    ap.add_argument("--dim", type=int, default=256)
    ap.add_argument("--dilation", type=int, default=1)
    ap.add_argument("--offset", type=int, default=0)
    ap.add_argument("--dtype", default="fp16", choices=["fp16", "bf16"])
    ap.add_argument("--stage", default="all", choices=("all",) + STAGES)
    ap.add_argument("--plan", default="tc", choices=["tc", "simt"])
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--profile", action="store_true")
    a = ap.parse_args()
    if a.op == "fscm":
        return fscm_main(a)

    dev = torch.device("cuda")
    dt = torch.float16 if a.dtype == "fp16" else torch.bfloat16
    B, T, D, N, K, dil, off = a.batch, a.seq, a.dim, a.basis, a.taps, a.dilation, a.offset
    L = off + T
    plan = capi.PLAN_TC if a.plan == "tc" else capi.PLAN_SIMT
    gen = torch.Generator(device=dev).manual_seed(0)
    nsets = 1 if a.profile else 2

    def make():
        return (torch.randn(B, D, L, device=dev, generator=gen).to(dt),
                (torch.randn(B, K, N, T, device=dev, generator=gen) * N ** -0.5).to(dt),
                (torch.randn(D, N, device=dev, generator=gen) * 3 ** -0.5).to(dt),
                torch.randn(B, D, T, device=dev, generator=gen).to(dt))

    sets = [make() for _ in range(nsets)]
    out = torch.empty(B, D, T, device=dev, dtype=dt)
    gh = torch.empty(B, D, L, device=dev, dtype=dt)
    gk = torch.empty(B, K, N, T, device=dev, dtype=dt)
    gm = torch.empty(D, N, device=dev, dtype=dt)
    h0, k0 = sets[0][0], sets[0][1]
    ws = torch.empty(max(256, capi.fdc_backward_workspace_size(h0, k0, off, dil, plan)),
                     dtype=torch.uint8, device=dev)

    def launch(stage, i):
        h, kc, mix, go = sets[i % nsets]
        if stage == "forward":
            capi.fdc_forward(h, kc, mix, out, off, dil, plan)
        elif stage == "grad_h":
            capi.fdc_backward_grad_h(go, kc, mix, gh, off, dil, plan)
        else:
            capi.fdc_backward_grad_kc_mix(go, h, kc, mix, gk, gm, ws, off, dil, plan)

    stages = STAGES if a.stage == "all" else (a.stage,)
    if a.profile:
        for i in range(4):
            launch(stages[0], i)
        torch.cuda.synchronize()
        print(json.dumps({"profile_launches": 4, "stage": stages[0],
                          "device_error": capi.device_error_info()}))
        return
    res = {"batch": B, "seq": T, "D": D, "N": N, "K": K, "dilation": dil, "offset": off,
           "dtype": a.dtype, "plan": a.plan}
    for st in stages:
        for i in range(5):
            launch(st, i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(a.iters):
            launch(st, i)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / a.iters * 1e3
        res[st] = {"us": us, "GB/s": algorithmic_bytes(st, B, T, D, N, K) / us / 1e3}
    res["device_error"] = capi.device_error_info()
    print(json.dumps(res))


if __name__ == "__main__":
    main()
