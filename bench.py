"""bench.py -- fused dynamic conv fwd+bwd throughput on B200 (one JSON line on rank 0).

Workload (BASELINE config 1 at N=128, the north-star shape): B=16 sequences per GPU,
T=L=4096 tokens, D=256 channels, K=3 taps, N=128 basis entries, dilation 1, t_offset 0,
fp16 inputs with fp32 accumulation; synthetic seeded inputs with the BASELINE
distributions (h, grad_out ~ N(0,1); kernel_chunk ~ N(0,1/N); kernel_mix ~ N(0,1/3)).
A step = forward + full backward (grad_h, grad_kernel_chunk, grad_kernel_mix) of one
batch, plus the sum of grad_kernel_mix over ranks when N>1 (data parallel over
independent sequences, B fixed per GPU: weak scaling; `--exchange` picks how: by default
inside the backward's last kernel over NVLink peer memory, delivered one step later, the
last step's sum inside the timed region).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --op fscm [--channels C] [--dilation d]     # source conv, 1 GPU

`value` is device time (CUDA events on the launching stream, max over ranks) with
inputs resident in HBM; two input sets rotate so every step streams >L2 (the
working set is ~460 MB against a 126 MB L2). `e2e` is the same metric through the
public drop-in API (`fused_dynamic_conv_chunk` + autograd backward) with pinned host
buffers: the H2D copies of the inputs and the D2H copies of the output and all three
gradients sit inside its timed region. `--impl reference` times the reference's CPU
algorithm (the numpy restatement in oracle/, all host threads) on a bounded sample of
the same workload. `roofline` describes the dominant kernel against the pipe whose minimum
time is longer (HBM bytes at the measured copy bandwidth, or tensor FLOPs at the measured
bf16 peak), with the other pipe's fraction beside it.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd tokens/s at D=256 K=3 N=128"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_TFLOPS = 1590.0  # bf16 dense, burst (cuBLAS), earlier measurement on this pool


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=16, help="sequences per GPU")
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--basis", type=int, default=128, help="N")
    ap.add_argument("--dilation", type=int, default=1)
    ap.add_argument("--dtype", default="fp16", choices=["fp16", "bf16", "fp32"],
                    help="fp32 runs the CUDA-core plan (the reference's AMP training likely "
                         "feeds the op fp32 tensors); not the headline configuration")
    ap.add_argument("--e2e-steps", type=int, default=60)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--op", default="fdc", choices=["fdc", "fscm", "kgen"],
                    help="fdc: the headline dynamic conv; fscm: fused_source_conv_mixed "
                         "(BASELINE config 3), one GPU; kgen: the kernel generator's tail "
                         "(softmax over K + flip) feeding the op, fused vs PyTorch, one GPU")
    ap.add_argument("--channels", type=int, default=16, help="fscm: source channels C")
    ap.add_argument("--exchange", default="peer-deferred", choices=["peer", "peer-deferred", "nccl"],
                    help="N>1: how grad_mix is summed over ranks: 'peer' = inside the "
                         "backward's last kernel over NVLink peer memory "
                         "(dudy_fdc_backward_dp); 'peer-deferred' = the same kernel sums "
                         "the previous step's grad_mix, which every rank published a step "
                         "earlier (dudy_fdc_backward_dp_deferred; the last step's sum by "
                         "dudy_fdc_exchange_finish inside the timed region); 'nccl' = a "
                         "torch.distributed all-reduce on a side stream, overlapping the "
                         "next step")
    ap.add_argument("--strong", action="store_true",
                    help="strong scaling: --batch is the global batch, split over the GPUs")
    ap.add_argument("--chunk", type=int, default=0,
                    help="fdc: time the model's call pattern instead: each step walks the "
                         "--seq tokens in calls of this many tokens (t_offset = c * chunk), "
                         "forward + backward per call, one GPU")
    return ap.parse_args()


def per_gpu_batch(a, world):
    if a.strong:
        if a.batch % world:
            raise SystemExit(f"--strong needs --batch ({a.batch}) divisible by {world}")
        return a.batch // world
    return a.batch


def config_dict(a, world):
    bpg = per_gpu_batch(a, world)
    return {
        "workload": "fused_dynamic_conv fwd+bwd, BASELINE config 1 (N=128)",
        "batch_per_gpu": bpg, "global_batch": bpg * world, "seq_len": a.seq,
        "D": 256, "K": 3, "N": a.basis, "dilation": a.dilation, "t_offset": 0,
        "parallelism": f"dp{world}" if world > 1 else "single",
        "grad_mix_exchange": {
            "peer": "peer memory inside the backward's last kernel (dudy_fdc_backward_dp)",
            "peer-deferred": "peer memory inside the next step's backward's last kernel "
                             "(dudy_fdc_backward_dp_deferred + dudy_fdc_exchange_finish)",
            "nccl": "NCCL all-reduce on a side stream"}[a.exchange] if world > 1 else None,
        "l2": "inputs larger than L2: two rotating input sets (~460 MB working set)",
    }


# ---------------------------------------------------------------------------------------
# algorithmic bytes per launch (fp16, per token x tokens per launch)
# ---------------------------------------------------------------------------------------
def step_roofline(B, T, D, N, K, step_ms, peak, peak_src, es=2):
    """The whole fwd+bwd step against HBM, per GPU: forward (2BTD + BTKN + DN) x es bytes
    (read h, kc, mix; write out) plus backward (3BTD + 2BTKN + 2DN) x es (read go, h, kc,
    mix; write grad_h, grad_kc, grad_mix), the minimum traffic of the op."""
    bt = B * T
    step_bytes = ((2 * bt * D + bt * K * N + D * N) + (3 * bt * D + 2 * bt * K * N + 2 * D * N)) * es
    achieved = step_bytes / (step_ms / 1e3) / 1e9
    return {"bound": "hbm", "algorithmic_bytes_per_step": step_bytes, "achieved": achieved,
            "peak": peak, "peak_source": peak_src, "unit": "GB/s", "frac": achieved / peak}


def algorithmic_bytes(B, T, D, N, K, es=2):
    bt = B * T
    conv = (bt * D + bt * K * N + D * N + bt * D) * es
    bk = (2 * bt * D + 2 * bt * K * N + 2 * D * N) * es
    return {
        # forward: read h, kc, mix; write out
        "fdc_tc_conv_kernel<forward>": conv,
        # grad_h: read go, kc, mix; write grad_h (either conv kernel)
        "fdc_tc_conv_kernel<grad_h>": conv,
        "fdc_tc_conv2_kernel<grad_h>": conv,
        # grad_kc + grad_mix: read go, h, kc, mix; write grad_kc, grad_mix
        "fdc_tc_bk_kernel": bk,
        "fdc_tc_bk_n128_kernel": bk,
    }


def algorithmic_flops(B, T, D, N, K):
    """Tensor-core FLOPs per launch of the tensor-core kernels: the per-token kernel
    W = kc . mix (2 B T K N D) in the forward and in grad_h; in the grad_kc/grad_mix kernels
    grad_mix = G . kc^T and grad_kc = mix^T . G, each contracted over both 16-bit terms of
    the exact product G = go*h (4 x 2 B T K N D)."""
    w = 2 * B * T * K * N * D
    return {
        "fdc_tc_conv_kernel<forward>": w,
        "fdc_tc_conv_kernel<grad_h>": w,
        "fdc_tc_conv2_kernel<grad_h>": w,
        "fdc_tc_bk_kernel": 4 * w,
        "fdc_tc_bk_n128_kernel": 4 * w,
    }


def kernel_bound(nbytes, flops, hbm_gbs, tensor_tflops):
    """The pipe that bounds a kernel: "tensor" when its FLOPs at the tensor peak take longer
    than its bytes at the HBM bandwidth, else "hbm" (no tensor work: "hbm")."""
    if flops is None:
        return "hbm"
    return "tensor" if flops / (tensor_tflops * 1e12) > nbytes / (hbm_gbs * 1e9) else "hbm"


def tc_kernel_names(D, N, K, dil):
    """The tensor-core kernel each stage runs, by the library's dispatch rule: grad_h uses
    the all-channel kernel when D is 128/256 and a tap start is not 8-token aligned, and the
    backward uses the TMEM-resident-mix kernel when N = 128."""
    shifted = any((kk * dil) % 8 for kk in range(1, K))
    gh = ("fdc_tc_conv2_kernel<grad_h>" if shifted and D in (128, 256)
          else "fdc_tc_conv_kernel<grad_h>")
    bk = "fdc_tc_bk_n128_kernel" if N == 128 and D in (128, 256) else "fdc_tc_bk_kernel"
    return ["fdc_tc_conv_kernel<forward>", gh, bk]


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def load_tensor_peak():
    """Dense bf16/fp16 tensor peak (TFLOP/s): the burst figure of MEASURED_PEAKS.json (the
    bench's kernels are timed over well under a second), else the fallback."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (burst)"
    except Exception:
        return FALLBACK_TFLOPS, "fallback"


def profiled_traffic(kernel: str):
    """DRAM bytes per launch from the committed ncu summary of this kernel, if any."""
    key = kernel.split("<")[0]
    suffix = "grad_h" if "grad_h" in kernel else ("forward" if "forward" in kernel else "")
    name = f"{key}{'_' + suffix if suffix else ''}_b16_t4096_n128.md"
    path = os.path.join(ROOT, "profiles", name)
    try:
        text = open(path).read()
    except OSError:
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", text)
    return float(m.group(1)) if m else None


# ---------------------------------------------------------------------------------------
# clocks sampled during the run
# ---------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_s: float = 0.01):
        self.gpu = gpu_index
        self.period = period_s
        self.rows = []
        self.proc = None
        self.thread = None
        self.source = None
        self._halt = threading.Event()

    def start(self):
        """Poll NVML (the counters nvidia-smi prints) every ``period`` seconds on a thread, so
        that a timed region of a fraction of a second still holds tens of samples; fall back
        to an ``nvidia-smi -lms 100`` process where NVML cannot be opened. Both only read.
        With no known GPU index nothing is sampled (the record says "unsampled")."""
        if self.gpu is None:
            self.source = "unsampled"
            return
        try:
            import pynvml
            pynvml.nvmlInit()
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.thread = threading.Thread(target=self._poll_nvml, args=(pynvml, handle),
                                           daemon=True)
            self.source = "nvml"
            self.thread.start()
            return
        except Exception:
            self.thread = None
        self.source = "nvidia-smi"
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def wait_first_sample(self, timeout_s: float):
        t0 = time.time()
        while self.thread is not None and not self.rows and time.time() - t0 < timeout_s:
            time.sleep(0.05)

    def _poll_nvml(self, nvml, handle):
        bits = (nvml.nvmlClocksEventReasonHwSlowdown, nvml.nvmlClocksEventReasonHwThermalSlowdown,
                nvml.nvmlClocksEventReasonSwThermalSlowdown, nvml.nvmlClocksEventReasonSwPowerCap)
        try:
            mx = nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM)
            while not self._halt.is_set():
                sm = nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM)
                pw = nvml.nvmlDeviceGetPowerUsage(handle) / 1e3
                rs = nvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                flags = ["Active" if rs & b else "Not Active" for b in bits]
                self.rows.append((time.time(), [str(self.gpu), str(sm), str(mx), f"{pw:.1f}",
                                                hex(rs), *flags]))
                self._halt.wait(self.period)
        except Exception:
            pass
        finally:
            try:
                nvml.nvmlShutdown()
            except Exception:
                pass

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append((time.time(), parts))

    def stop(self):
        self._halt.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0=None, t1=None):
        rows = [r for (t, r) in self.rows if (t0 is None or t >= t0) and (t1 is None or t <= t1)]
        if not rows:
            rows = [r for (_, r) in self.rows]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0,
                    "source": self.source}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1])]
        mx = [num(r[2]) for r in rows if num(r[2])]
        pw = [num(r[3]) for r in rows if num(r[3])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None,
                "reasons": reasons, "samples": len(rows), "source": self.source}


def physical_gpu(local_rank: int):
    """NVML index of this process's GPU, or None when it cannot be told for certain.

    Resolved through the device's UUID (torch's device properties against NVML), which
    holds whatever CUDA_VISIBLE_DEVICES contains (indices, UUIDs or MIG names); a plain
    index list is the fallback. None means the clock record reports "unsampled" rather than
    another GPU's counters."""
    try:
        import pynvml
        import torch

        uuid = str(torch.cuda.get_device_properties(local_rank).uuid)
        pynvml.nvmlInit()
        try:
            for i in range(pynvml.nvmlDeviceGetCount()):
                u = pynvml.nvmlDeviceGetUUID(pynvml.nvmlDeviceGetHandleByIndex(i))
                u = u.decode() if isinstance(u, bytes) else u
                if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                    return i
        finally:
            pynvml.nvmlShutdown()
    except Exception:
        pass
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if not vis:
        return local_rank
    parts = vis.split(",")
    if local_rank < len(parts) and parts[local_rank].strip().isdigit():
        return int(parts[local_rank])
    return None


# ---------------------------------------------------------------------------------------
# CPU baseline: the reference's algorithm (numpy restatement), bounded sample
# ---------------------------------------------------------------------------------------
def cpu_baseline(a, seconds: float):
    import numpy as np

    from oracle import fdc_forward_backward_fp32

    rng = np.random.Generator(np.random.PCG64(0))
    B, T, D, N, K = 1, a.seq, 256, a.basis, 3
    h = rng.standard_normal((B, D, T), dtype=np.float32)
    kc = rng.standard_normal((B, K, N, T), dtype=np.float32) * np.float32(N ** -0.5)
    mix = rng.standard_normal((D, N), dtype=np.float32) * np.float32(3 ** -0.5)
    go = rng.standard_normal((B, D, T), dtype=np.float32)
    fdc_forward_backward_fp32(h, kc, mix, go, 0, a.dilation)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        fdc_forward_backward_fp32(h, kc, mix, go, 0, a.dilation)
        n += 1
        el = time.perf_counter() - t0
        if (el >= seconds and n >= 2) or n >= 1000:
            break
    return {"value": B * T * n / el, "unit": UNIT, "cores": os.cpu_count(),
            "kind": "port",
            "sample": f"{n} fwd+bwd passes of 1 sequence x {T} tokens (D=256, K=3, N={N}, "
                      f"fp32, numpy restatement of the reference's torch formula) in {el:.1f} s"}


# B=2, T=512, D=256, N=16, K=3, dilation 1, fp32, seed 0
CFG0 = dict(B=2, T=512, D=256, N=16, K=3, dil=1)


def config0_inputs():
    import numpy as np
    rng = np.random.Generator(np.random.PCG64(0))
    B, T, D, N, K = (CFG0[k] for k in ("B", "T", "D", "N", "K"))
    h = rng.standard_normal((B, D, T), dtype=np.float32)
    kc = rng.standard_normal((B, K, N, T), dtype=np.float32) * np.float32(N ** -0.5)
    mix = rng.standard_normal((D, N), dtype=np.float32) * np.float32(3 ** -0.5)
    go = rng.standard_normal((B, D, T), dtype=np.float32)
    return h, kc, mix, go


def config0_cpu():
    """BASELINE config 0 on the host: the reference's CPU formula (numpy restatement, fp32,
    all host threads), median of 5 fwd+bwd passes after 2 warm-ups."""
    from oracle import fdc_forward_backward_fp32
    h, kc, mix, go = config0_inputs()
    times = []
    for i in range(7):
        t0 = time.perf_counter()
        fdc_forward_backward_fp32(h, kc, mix, go, 0, CFG0["dil"])
        if i >= 2:
            times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": CFG0["B"] * CFG0["T"] / med, "unit": UNIT, "ms_per_step": 1e3 * med,
            "cores": os.cpu_count(), "kind": "port",
            "sample": "BASELINE config 0 (B=2, T=512, D=256, N=16, K=3, dilation 1, fp32, "
                      "seed 0), median of 5 fwd+bwd passes after 2 warm-ups"}


def config0_gpu(dev):
    """BASELINE config 0 on one GPU through the C ABI (fp32: the CUDA-core plan), inputs
    resident, CUDA events around each fwd+bwd pass, median of 20 after 3 warm-ups."""
    import torch

    from dudyconv_b200 import capi
    h, kc, mix, go = (torch.from_numpy(x).to(dev) for x in config0_inputs())
    off, dil = 0, CFG0["dil"]
    out, gh, gk, gm = (torch.empty_like(x) for x in (go, h, kc, mix))
    ws = torch.empty(max(256, capi.fdc_backward_workspace_size(h, kc, off, dil)),
                     dtype=torch.uint8, device=dev)
    times = []
    for i in range(23):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        capi.fdc_forward(h, kc, mix, out, off, dil)
        capi.fdc_backward(go, h, kc, mix, gh, gk, gm, ws, off, dil)
        e1.record()
        torch.cuda.synchronize()
        if i >= 3:
            times.append(e0.elapsed_time(e1))
    med = statistics.median(times)
    plan = capi.fdc_default_plan(h, kc, mix, off, dil)
    return {"value": CFG0["B"] * CFG0["T"] / (med / 1e3), "unit": UNIT, "ms_per_step": med,
            "dtype": "f32", "plan": capi.lib().dudy_fdc_plan_name(plan).decode(),
            "sample": "BASELINE config 0 through the C ABI, inputs resident, median of 20 "
                      "fwd+bwd passes after 3 warm-ups"}


def run_reference(a, world, rank):
    if rank != 0:
        return
    steps = []
    import numpy as np

    from oracle import fdc_forward_backward_fp32
    rng = np.random.Generator(np.random.PCG64(1))
    B, T, D, N, K = 1, a.seq, 256, a.basis, 3
    h = rng.standard_normal((B, D, T), dtype=np.float32)
    kc = rng.standard_normal((B, K, N, T), dtype=np.float32) * np.float32(N ** -0.5)
    mix = rng.standard_normal((D, N), dtype=np.float32) * np.float32(3 ** -0.5)
    go = rng.standard_normal((B, D, T), dtype=np.float32)
    for i in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        fdc_forward_backward_fp32(h, kc, mix, go, 0, a.dilation)
        if i >= a.warmup:
            steps.append(time.perf_counter() - t0)
    total = sum(steps)
    value = B * T * len(steps) / total
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * total / len(steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config_dict(a, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                         "sample": f"each step = 1 sequence x {T} tokens fwd+bwd (of the "
                                   f"{a.batch}-sequence batch), numpy restatement of the "
                                   f"reference's CPU torch formula, all host threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "config0": config0_cpu(),
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------
def run_ours(a, world, rank, local_rank):
    import torch
    import torch.distributed as dist

    from dudyconv_b200 import capi
    from dudyconv_b200.dp import allreduce_grad_mix

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dt = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[a.dtype]
    B, T, D, N, K, dil, off = per_gpu_batch(a, world), a.seq, 256, a.basis, 3, a.dilation, 0
    L = T
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)

    def make_set():
        h = torch.randn(B, D, L, device=dev, generator=gen).to(dt)
        kc = (torch.randn(B, K, N, T, device=dev, generator=gen) * N ** -0.5).to(dt)
        mix = (torch.randn(D, N, device=dev, generator=gen) * 3 ** -0.5).to(dt)
        go = torch.randn(B, D, T, device=dev, generator=gen).to(dt)
        return h, kc, mix, go

    sets = [make_set(), make_set()]
    out = torch.empty(B, D, T, device=dev, dtype=dt)
    gh = torch.empty(B, D, L, device=dev, dtype=dt)
    gk = torch.empty(B, K, N, T, device=dev, dtype=dt)
    gm = torch.empty(D, N, device=dev, dtype=dt)
    plan = capi.fdc_default_plan(sets[0][0], sets[0][1], sets[0][2], off, dil)
    ws = torch.empty(max(256, capi.fdc_backward_workspace_size(sets[0][0], sets[0][1], off, dil)),
                     dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    kernels = (tc_kernel_names(D, N, K, dil)
               if plan == capi.PLAN_TC else
               ["fdc_conv_simt_kernel<forward>", "fdc_conv_simt_kernel<grad_h>",
                "fdc_grad_kc_simt_kernel+fdc_grad_mix_*"])
    launches_per_step = 4 if plan == capi.PLAN_TC else 5

    # N > 1, exchange "peer": the backward's last kernel sums grad_mix over the ranks
    # through peer memory (dudy_fdc_backward_dp), in the step itself.
    # N > 1, exchange "peer-deferred": the same kernel publishes step i's sums and adds up
    # step i-1's (published by every rank a step earlier); the last step's sum comes from a
    # finish launch inside the timed region.
    # N > 1, exchange "nccl": the grad_mix all-reduce of step i runs on its own stream while
    # step i+1 computes; grad_mix is double-buffered and step i+2 waits until the exchange
    # of step i has finished with it
    peer = world > 1 and a.exchange in ("peer", "peer-deferred")
    deferred = peer and a.exchange == "peer-deferred"
    gm_sum = torch.empty_like(gm)  # deferred: the previous step's sum over ranks
    xch = None
    if peer:
        from dudyconv_b200.dp import GradMixExchange
        xch = GradMixExchange(D, N, device=dev)
    gms = [gm, torch.empty_like(gm)]
    s_comm = torch.cuda.Stream(dev) if world > 1 and not peer else None
    comm_done = [torch.cuda.Event(), torch.cuda.Event()]
    comm_used = [False, False]

    def step(i, evs=None):
        h, kc, mix, go = sets[i & 1]
        gm = gms[i & 1]
        if s_comm is not None and comm_used[i & 1]:
            stream.wait_event(comm_done[i & 1])
        if evs is None:
            # the reference's two calls: forward, then the whole backward
            capi.fdc_forward(h, kc, mix, out, off, dil, plan)
            if deferred:
                xch.backward_deferred(go, h, kc, mix, gh, gk, gm, gm_sum, ws, off, dil, plan)
            elif peer:
                xch.backward(go, h, kc, mix, gh, gk, gm, ws, off, dil, plan)
            else:
                capi.fdc_backward(go, h, kc, mix, gh, gk, gm, ws, off, dil, plan)
        else:
            # per-kernel pass: the backward's two parts as separate calls, events between
            evs[0].record(stream)
            capi.fdc_forward(h, kc, mix, out, off, dil, plan)
            evs[1].record(stream)
            capi.fdc_backward_grad_h(go, kc, mix, gh, off, dil, plan)
            evs[2].record(stream)
            capi.fdc_backward_grad_kc_mix(go, h, kc, mix, gk, gm, ws, off, dil, plan)
            evs[3].record(stream)
            return  # per-kernel pass: this rank's kernels only, no exchange
        if s_comm is not None:
            bwd_done = torch.cuda.Event()
            bwd_done.record(stream)
            s_comm.wait_event(bwd_done)
            with torch.cuda.stream(s_comm):
                allreduce_grad_mix(gm)
            comm_done[i & 1].record(s_comm)
            comm_used[i & 1] = True

    clocks = ClockSampler(physical_gpu(local_rank))
    if rank == 0:
        clocks.start()
        clocks.wait_first_sample(10.0)  # keep nvidia-smi start-up out of the timed region
    for i in range(a.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # headline: K steps back to back, events only around the whole region (an event
    # between two kernels would also stop the programmatic-launch overlap of the next one)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    t_start.record(stream)
    for i in range(a.steps):
        step(i)
    if s_comm is not None:
        stream.wait_stream(s_comm)  # the last exchanges are inside the timed region
    if deferred:
        xch.finish(gm_sum)  # the last step's sum, inside the timed region
    t_end.record(stream)
    torch.cuda.synchronize()
    wall1 = time.time()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = t_start.elapsed_time(t_end)
    # per-kernel durations for the roofline: the same K steps again, with an event pair
    # around every kernel on the launching stream
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(a.steps)]
    for i in range(a.steps):
        step(i, evs[i])
    torch.cuda.synchronize()
    seg = [0.0, 0.0, 0.0]
    for e in evs:
        for j in range(3):
            seg[j] += e[j].elapsed_time(e[j + 1])
    # peer exchange: the backward with the exchange, timed alone per step (events around the
    # whole call), against the same backward without it
    bwd_dp = None
    if peer:
        pairs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(a.steps)]
        for i in range(a.steps):
            h_, kc_, mix_, go_ = sets[i & 1]
            pairs[i][0].record(stream)
            capi.fdc_backward(go_, h_, kc_, mix_, gh, gk, gms[i & 1], ws, off, dil, plan)
            pairs[i][1].record(stream)
            pairs[i][2].record(stream)
            if deferred:
                xch.backward_deferred(go_, h_, kc_, mix_, gh, gk, gms[i & 1], gm_sum, ws, off,
                                      dil, plan)
            else:
                xch.backward(go_, h_, kc_, mix_, gh, gk, gms[i & 1], ws, off, dil, plan)
            pairs[i][3].record(stream)
        torch.cuda.synchronize()
        bwd_dp = {"backward_ms": sum(p_[0].elapsed_time(p_[1]) for p_ in pairs) / a.steps,
                  "backward_with_exchange_ms":
                      sum(p_[2].elapsed_time(p_[3]) for p_ in pairs) / a.steps}
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    assert capi.device_error() == 0, "tensor-core kernel reported a wait timeout"

    # e2e: public drop-in API, pinned host buffers, copies inside the timed region. Copies
    # are double-buffered on their own streams, as a training input pipeline would run
    # them: step i+1's inputs upload while step i computes and step i-1's results
    # download (H2D and D2H use the two directions of the host link at once).
    e2e = None
    if not a.no_e2e:
        import dudyconv_b200.cuda_ops as co
        hs = [x.cpu().pin_memory() for x in sets[0]]
        outs = [torch.empty(s, dtype=dt).pin_memory() for s in ((B, D, T), (B, D, L), (B, K, N, T), (D, N))]
        h2d = sum(x.numel() * x.element_size() for x in hs)
        d2h = sum(x.numel() * x.element_size() for x in outs)
        s_in = torch.cuda.Stream(dev)
        s_out = torch.cuda.Stream(dev)
        dev_in = [[torch.empty_like(x, device=dev) for x in hs] for _ in range(2)]
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [torch.cuda.Event() for _ in range(2)]

        def e2e_step(i):
            slot = i & 1
            with torch.cuda.stream(s_in):
                s_in.wait_event(in_free[slot])  # step i-2 is done reading this slot
                for d_, h_ in zip(dev_in[slot], hs):
                    d_.copy_(h_, non_blocking=True)
                in_ready[slot].record(s_in)
            stream.wait_event(in_ready[slot])
            h, kc, mix, go = (t.detach() for t in dev_in[slot])
            h.requires_grad_(True)
            kc.requires_grad_(True)
            mix.requires_grad_(True)
            y = co.fused_dynamic_conv_chunk(h, kc, mix, 0, dil)
            y.backward(go)
            if world > 1:
                allreduce_grad_mix(mix.grad)
            in_free[slot].record(stream)
            done = torch.cuda.Event()
            done.record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                for dst, src in zip(outs, (y, h.grad, kc.grad, mix.grad)):
                    src.record_stream(s_out)
                    dst.copy_(src.detach(), non_blocking=True)

        for i in range(3):
            e2e_step(i)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_event(e0)
        for i in range(a.e2e_steps):
            e2e_step(i)
        e1.record(s_out)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([e_ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": B * T * world * a.e2e_steps / (e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "dudyconv_b200.cuda_ops.fused_dynamic_conv_chunk + autograd backward",
               "copies": "pinned host buffers; H2D and D2H on their own streams, double-buffered "
                         "device inputs, all inside the timed region"}
    if rank == 0:
        clocks.stop()
    if world > 1:
        dist.barrier()
    if rank != 0:
        return

    tokens = B * T * world * a.steps
    value = tokens / (ms / 1e3)
    es = 4 if a.dtype == "fp32" else 2
    alg = algorithmic_bytes(B, T, D, N, K, es)
    shares = [s / max(sum(seg), 1e-12) for s in seg]
    dom = max(range(3), key=lambda j: seg[j])
    dom_name = kernels[dom]
    avg_ms = seg[dom] / a.steps
    peak, peak_src = load_peaks()
    tpeak, tpeak_src = load_tensor_peak()
    flops = algorithmic_flops(B, T, D, N, K) if plan == capi.PLAN_TC else {}
    roof = None
    if dom_name in alg:
        # the bound is the pipe whose minimum time is longer: HBM (algorithmic bytes at the
        # measured copy bandwidth) or the tensor cores (algorithmic FLOPs at the measured
        # bf16 peak); the exact-product grad_kc/grad_mix kernel (51.5 GFLOP, 168 MB at the
        # hot shape) is tensor-bound
        hbm_ach = alg[dom_name] / (avg_ms / 1e3) / 1e9
        f = flops.get(dom_name)
        tensor_bound = kernel_bound(alg[dom_name], f, peak, tpeak) == "tensor"
        common = {"kernel": dom_name, "algorithmic_bytes_per_launch": alg[dom_name],
                  "algorithmic_flops_per_launch": f, "avg_launch_ms": avg_ms,
                  "traffic": profiled_traffic(dom_name),
                  "hbm": {"achieved": hbm_ach, "peak": peak, "unit": "GB/s",
                          "frac": hbm_ach / peak, "peak_source": peak_src},
                  "timing": "CUDA events around each launch, K extra steps after the headline "
                            "region (events between kernels disable the launch overlap)"}
        if tensor_bound:
            t_ach = f / (avg_ms / 1e3) / 1e12
            roof = {"bound": "tensor", "achieved": t_ach, "peak": tpeak, "unit": "TFLOP/s",
                    "frac": t_ach / tpeak, "peak_source": tpeak_src, **common}
        else:
            roof = {"bound": "hbm", "achieved": hbm_ach, "peak": peak, "unit": "GB/s",
                    "frac": hbm_ach / peak, "peak_source": peak_src, **common}
    per_kernel = {kernels[j]: {"avg_ms": seg[j] / a.steps, "share": shares[j],
                               "achieved_gbs": (alg[kernels[j]] / (seg[j] / a.steps / 1e3) / 1e9)
                               if kernels[j] in alg else None}
                  for j in range(3)}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True,
        "scaling": "strong" if a.strong else "weak", "vs_baseline": None,
        "dtype": {"fp16": "f16", "bf16": "bf16", "fp32": "f32"}[a.dtype],
        "data": "synthetic (seeded, BASELINE distributions)", "config": config_dict(a, world),
        "plan": capi.lib().dudy_fdc_plan_name(plan).decode(),
        "roofline": roof, "per_kernel": per_kernel, "exchange_timing": bwd_dp,
        "step_roofline": step_roofline(B, T, D, N, K, ms / a.steps, peak, peak_src, es),
        "clocks": clocks.summary(wall0, wall1),
        "gpu_launches": launches_per_step * a.steps + (1 if deferred else 0),
        "e2e": e2e,
    }
    if world == 1:
        line["config0"] = {"gpu": config0_gpu(dev)}
        if not a.no_cpu_baseline:
            line["config0"]["cpu"] = config0_cpu()
    if world == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(a, a.cpu_seconds)
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------
# source conv (fused_source_conv_mixed): one GPU
# ---------------------------------------------------------------------------------------
def run_fscm(a, rank):
    """fwd+bwd of the source conv at B=16, T=4096, D=256, S=3, C channels, one dilation.
    The op is bound by its C erf-GELU evaluations per (token, channel) at C = 16 (FP32 /
    SFU issue), so the line reports GELU evaluations per second next to the HBM
    fraction of its algorithmic bytes."""
    if rank != 0:
        return
    import numpy as np
    import torch

    from dudyconv_b200 import capi

    dev = torch.device("cuda")
    dt = torch.float16 if a.dtype == "fp16" else torch.bfloat16
    B, T, D, C, S, dil = a.batch, a.seq, 256, a.channels, 3, a.dilation
    gen = torch.Generator(device=dev).manual_seed(2024)

    def make():
        return (torch.randn(B, D, T, device=dev, generator=gen).to(dt),
                (torch.randn(D, C, S, device=dev, generator=gen) * 3 ** -0.5).to(dt),
                (torch.randn(D, C, device=dev, generator=gen) * C ** -0.5).to(dt),
                (torch.randn(D, C, device=dev, generator=gen) * C ** -0.5).to(dt),
                torch.zeros(D, device=dev, dtype=dt),
                torch.randn(B, D, T, device=dev, generator=gen).to(dt))

    sets = [make(), make()]
    out = torch.empty(B, D, T, device=dev, dtype=dt)
    gx = torch.empty_like(sets[0][0])
    gw = torch.empty_like(sets[0][1])
    gb = torch.empty(D, C, device=dev, dtype=dt)
    gmw = torch.empty(D, C, device=dev, dtype=dt)
    gmb = torch.empty(D, device=dev, dtype=dt)
    ws = torch.empty(max(256, capi.fscm_backward_workspace_size(sets[0][0], sets[0][1], 0, T,
                                                                dil)),
                     dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def step(i, evs=None):
        x, w, bias, mw, mb, go = sets[i & 1]
        if evs:
            evs[0].record(stream)
        capi.fscm_forward(x, w, bias, mw, mb, out, 0, T, dil)
        if evs:
            evs[1].record(stream)
        capi.fscm_backward(go, x, w, bias, mw, mb, gx, gw, gb, gmw, gmb, ws, 0, T, dil)
        if evs:
            evs[2].record(stream)

    clocks = ClockSampler(physical_gpu(0))
    clocks.start()
    clocks.wait_first_sample(10.0)
    for i in range(a.warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    e0.record(stream)
    for i in range(a.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    wall1 = time.time()
    clocks.stop()
    ms = e0.elapsed_time(e1) / a.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(a.steps)]
    for i in range(a.steps):
        step(i, evs[i])
    torch.cuda.synchronize()
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / a.steps
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / a.steps
    assert capi.device_error() == 0
    bt = B * T
    alg = {"forward": 2 * bt * D * 2, "backward": 3 * bt * D * 2}
    peak, peak_src = load_peaks()
    gelus = bt * D * C
    # CPU baseline: the reference formula (numpy restatement), one sequence per pass
    rng = np.random.Generator(np.random.PCG64(0))
    xs = rng.standard_normal((1, D, T)).astype(np.float32)
    wv = (rng.standard_normal((D, C, S)) * 3 ** -0.5).astype(np.float32)
    bv = (rng.standard_normal((D, C)) * C ** -0.5).astype(np.float32)
    mwv = (rng.standard_normal((D, C)) * C ** -0.5).astype(np.float32)
    mbv = np.zeros(D, np.float32)
    gov = rng.standard_normal((1, D, T)).astype(np.float32)
    from oracle.fscm import fscm_backward as ref_bwd, fscm_forward as ref_fwd
    n, t0 = 0, time.perf_counter()
    while True:
        ref_fwd(xs, wv, bv, mwv, mbv, 0, T, dil, dtype=np.float32)
        ref_bwd(gov, xs, wv, bv, mwv, mbv, 0, T, dil, dtype=np.float32)
        n += 1
        el = time.perf_counter() - t0
        if (el >= a.cpu_seconds and n >= 2) or n >= 200:
            break
    line = {
        "metric": f"fscm fwd+bwd tokens/s at D=256 S=3 C={C} dilation={dil}",
        "value": bt / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16" if a.dtype == "fp16" else "bf16",
        "data": "synthetic (seeded, BASELINE config 3 distributions)",
        "config": {"workload": "fused_source_conv_mixed fwd+bwd, BASELINE config 3",
                   "batch": B, "seq_len": T, "D": D, "S": S, "C": C, "dilation": dil,
                   "t_offset": 0, "l2": "two rotating input sets (2 x 67 MB)"},
        "roofline": {"kernel": "fscm_fwd_kernel + fscm_bwd_kernel", "bound": "hbm",
                     "achieved": (alg["forward"] + alg["backward"]) / ((fwd_ms + bwd_ms) / 1e3) / 1e9,
                     "peak": peak, "unit": "GB/s", "peak_source": peak_src,
                     "frac": (alg["forward"] + alg["backward"]) / ((fwd_ms + bwd_ms) / 1e3) / 1e9 / peak,
                     "traffic": None,
                     "note": "FP32/SFU issue-bound (C erf-GELU per token-channel), not HBM"},
        "per_kernel": {"forward_ms": fwd_ms, "backward_ms": bwd_ms,
                       "gelu_per_s_forward": gelus / (fwd_ms / 1e3),
                       "gelu_per_s_backward": gelus / (bwd_ms / 1e3)},
        "gpu_launches": 3 * a.steps,
        "clocks": clocks.summary(wall0, wall1),
        "cpu_baseline": {"value": T * n / el, "unit": UNIT, "cores": os.cpu_count(),
                         "kind": "port",
                         "sample": f"{n} fwd+bwd passes of 1 sequence x {T} tokens (fp32, numpy "
                                   f"restatement of the reference's torch formula) in {el:.1f} s"},
    }
    print(json.dumps(line), flush=True)


def run_kgen(a, rank):
    """The kernel generator's tail feeding the op (the model's per-chunk sequence
    logits -> _logits_to_kernel -> fused_dynamic_conv_chunk, forward + backward), at the
    headline shape: PyTorch's tail (softmax, flip copy, permute copy, backbone_dil_unshared.py:
    1821-1900) against the fused one-pass logits_to_kernel, both feeding this library's op.
    Reported: both chains' times, and the fused tail alone against its algorithmic bytes
    (forward: read logits, write kernel_chunk; backward: read kernel_chunk and its
    gradient, write the logits' gradient)."""
    if rank != 0:
        return
    import torch
    import torch.nn.functional as F

    import dudyconv_b200.cuda_ops as co
    from dudyconv_b200.kernel_gen import logits_to_kernel

    dev = torch.device("cuda")
    dt = torch.float16 if a.dtype == "fp16" else torch.bfloat16
    B, T, D, N, K = a.batch, a.seq, 256, a.basis, 3
    gen = torch.Generator(device=dev).manual_seed(77)
    h = torch.randn(B, D, T, device=dev, generator=gen).to(dt).requires_grad_(True)
    mix = (torch.randn(D, N, device=dev, generator=gen) * 3 ** -0.5).to(dt).requires_grad_(True)
    logits = (torch.randn(B, N * K, T, device=dev, generator=gen) * 1.5).to(dt).requires_grad_(True)
    go = torch.randn(B, D, T, device=dev, generator=gen).to(dt)
    gkc = torch.randn(B, K, N, T, device=dev, generator=gen).to(dt)

    def torch_tail(x):
        y = F.softmax(x.reshape(B, N, K, T), dim=2)
        return torch.flip(y, dims=[2]).permute(0, 2, 1, 3).contiguous()

    def tail_step(fn):
        kc = fn(logits)
        kc.backward(gkc)

    def chain_step(fn):
        kc = fn(logits)
        out = co.fused_dynamic_conv_chunk(h, kc, mix, 0, 1)
        out.backward(go)

    fused = lambda x: logits_to_kernel(x, N, K)  # noqa: E731

    def timed(step, fn, n):
        for _ in range(a.warmup):
            step(fn)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            step(fn)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    n = max(10, min(a.steps, 200))
    clocks = ClockSampler(physical_gpu(0))
    clocks.start()
    clocks.wait_first_sample(10.0)
    wall0 = time.time()
    t_tail_torch = timed(tail_step, torch_tail, n)
    t_tail_fused = timed(tail_step, fused, n)
    t_chain_torch = timed(chain_step, torch_tail, n)
    t_chain_fused = timed(chain_step, fused, n)
    wall1 = time.time()
    clocks.stop()
    elems = B * K * N * T
    es = 2
    tail_bytes_fused = elems * es * (2 + 3)   # fwd: read logits, write kc; bwd: kc, gkc -> gl
    peak, peak_src = load_peaks()
    ach = tail_bytes_fused / (t_tail_fused / 1e3) / 1e9
    print(json.dumps({
        "metric": "kernel-generator tail + op fwd+bwd tokens/s at D=256 K=3 N=128",
        "value": B * T / (t_chain_fused / 1e3), "unit": UNIT, "n_gpus": 1, "steps": n,
        "warmup": a.warmup, "ms_per_step": t_chain_fused, "higher_is_better": True,
        "dtype": a.dtype, "data": "synthetic (seeded)",
        "config": {"workload": "logits [B,N*K,T] -> kernel_chunk -> fused_dynamic_conv_chunk, "
                               "forward + backward", "batch": B, "seq_len": T, "N": N, "K": K},
        "torch_tail_chain": {"ms_per_step": t_chain_torch,
                             "tokens_per_s": B * T / (t_chain_torch / 1e3)},
        "tail_only": {"torch_ms": t_tail_torch, "fused_ms": t_tail_fused,
                      "fused_bytes": tail_bytes_fused,
                      "fused_roofline": {"bound": "hbm", "achieved": ach, "peak": peak,
                                         "unit": "GB/s", "frac": ach / peak,
                                         "peak_source": peak_src}},
        "gpu_launches": None, "clocks": clocks.summary(wall0, wall1)}), flush=True)


def run_chunked(a, rank):
    """The chunked call path of the model (the op called per `--chunk` tokens of a longer
    sequence with t_offset, grad_h returned full-length each call): forward + combined
    backward per chunk through the C ABI, one GPU; not the headline configuration."""
    import torch

    from dudyconv_b200 import capi

    if rank != 0:
        return
    dev = torch.device("cuda", 0)
    dt = torch.float16 if a.dtype == "fp16" else torch.bfloat16
    B, L, D, N, K, dil, C = a.batch, a.seq, 256, a.basis, 3, a.dilation, a.chunk
    nc = L // C
    gen = torch.Generator(device=dev).manual_seed(1234)
    h = torch.randn(B, D, L, device=dev, generator=gen).to(dt)
    mix = (torch.randn(D, N, device=dev, generator=gen) * 3 ** -0.5).to(dt)
    kcs = [(torch.randn(B, K, N, C, device=dev, generator=gen) * N ** -0.5).to(dt)
           for _ in range(nc)]
    gos = [torch.randn(B, D, C, device=dev, generator=gen).to(dt) for _ in range(nc)]
    out = torch.empty(B, D, C, device=dev, dtype=dt)
    gh = torch.empty(B, D, L, device=dev, dtype=dt)
    gk = torch.empty(B, K, N, C, device=dev, dtype=dt)
    gm = torch.empty(D, N, device=dev, dtype=dt)
    ws = torch.empty(max(256, capi.fdc_backward_workspace_size(h, kcs[0], 0, dil)),
                     dtype=torch.uint8, device=dev)

    def step():
        for c in range(nc):
            capi.fdc_forward(h, kcs[c], mix, out, c * C, dil)
            capi.fdc_backward(gos[c], h, kcs[c], mix, gh, gk, gm, ws, c * C, dil)

    clocks = ClockSampler(physical_gpu(0))
    clocks.start()
    clocks.wait_first_sample(10.0)
    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    e0.record()
    for _ in range(a.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    wall1 = time.time()
    clocks.stop()
    ms = e0.elapsed_time(e1) / a.steps
    assert capi.device_error() == 0, "tensor-core kernel reported a wait timeout"
    print(json.dumps({
        "metric": f"fwd+bwd tokens/s at D=256 K=3 N={N}, {C}-token chunked calls",
        "value": B * L / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "dtype": a.dtype,
        "data": "synthetic (seeded)",
        "config": {"workload": f"{nc} calls of {C} tokens per step (t_offset = c * {C}), "
                               f"forward + backward each, grad_h full-length [B,D,L]",
                   "batch": B, "seq_len": L, "chunk": C, "dilation": dil},
        "us_per_chunk": ms * 1e3 / nc, "clocks": clocks.summary(wall0, wall1)}), flush=True)


def main():
    a = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference(a, world, rank)
        return
    if a.op == "fscm":
        run_fscm(a, rank)
        return
    if a.op == "kgen":
        run_kgen(a, rank)
        return
    if a.chunk > 0:
        run_chunked(a, rank)
        return
    import torch.distributed as dist
    if world > 1:
        import datetime

        import torch
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(a, world, rank, local_rank)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
