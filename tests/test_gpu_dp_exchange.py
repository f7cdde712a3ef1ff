"""The data-parallel backward with the grad_mix sum over ranks in its last kernel.

Two to four ranks (as many as there are GPUs, at most four; skipped with fewer than two),
one GPU each, each with its own sequences:
``dudy_fdc_backward_dp`` must give every rank bitwise-identical grad_mix equal (within the
parity bar) to the float64 oracle's grad_mix summed over all ranks' sequences, leave
grad_h and grad_kc exactly as the plain backward computes them, and stay correct over
consecutive calls (the exchange's four slots and epoch counter) on the tensor-core
plan (fp16, bf16) and on the CUDA-core plan (fp32, with D*N not a multiple of 4). The
deferred form (``dudy_fdc_backward_dp_deferred`` + ``dudy_fdc_exchange_finish``), run on
the same inputs after the synchronous calls on the same buffers, must return this rank's
own grad_mix from each call and, one call later (the last one from the finish launch),
exactly the synchronous call's sum. The ranks run as spawned child processes with a
deadline; NVLS is off in NCCL.
"""

import os
import sys
import time

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu

CASES = [
    # (B, D, L, T, N, K, off, dil, dtype)
    (2, 256, 384, 384, 128, 3, 0, 1, "fp16"),
    (1, 256, 640, 512, 64, 3, 128, 2, "bf16"),
    (2, 17, 67, 19, 5, 4, 23, 2, "fp32"),
]


def _worker(rank, world, port, q):
    try:
        sys.path[:0] = [ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "tests", "golden")]
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        import datetime

        import numpy as np
        import torch.distributed as dist

        from dudyconv_b200 import capi
        from dudyconv_b200.dp import GradMixExchange
        from inputs import fdc_inputs
        from oracle import fdc_backward
        from parity import TORCH_DT, assert_close

        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        for ci, (B, D, L, T, N, K, off, dil, dt) in enumerate(CASES):
            xch = GradMixExchange(D, N)
            sums, calls = [], []
            for call in range(3):
                # rank-specific sequences; the third call repeats the first call's inputs
                seed = 100 * ci + 10 * rank + (call % 2)
                h, kc, mix, go = fdc_inputs([B, D, L, T, N, K, off, dil], dt, "base", seed)
                _, _, mix, _ = fdc_inputs([B, D, L, T, N, K, off, dil], dt, "base", 100 * ci)
                th, tk, tm, tg = (torch.from_numpy(np.ascontiguousarray(a)).to(
                    "cuda", TORCH_DT[dt]) for a in (h, kc, mix, go))
                ws = torch.empty(max(256, capi.fdc_backward_workspace_size(th, tk, off, dil)),
                                 dtype=torch.uint8, device="cuda")
                gh, gk, gm = (torch.full_like(x, float("nan")) for x in (th, tk, tm))
                xch.backward(tg, th, tk, tm, gh, gk, gm, ws, off, dil)
                ref = [torch.empty_like(x) for x in (th, tk, tm)]
                capi.fdc_backward(tg, th, tk, tm, *ref, ws, off, dil)
                torch.cuda.synchronize()
                assert capi.device_error() == 0, capi.device_error_info()
                assert torch.equal(gh, ref[0]) and torch.equal(gk, ref[1]), (ci, call)
                # bitwise-identical grad_mix on every rank
                allm = [torch.empty_like(gm) for _ in range(world)]
                dist.all_gather(allm, gm)
                for r in range(world):
                    assert torch.equal(allm[r], gm), (ci, call, r)
                # against the oracle summed over the ranks' sequences (float64)
                _, _, gm_loc = fdc_backward(go, h, kc, mix, off, dil)
                tot = torch.from_numpy(gm_loc).cuda()
                dist.all_reduce(tot)
                assert_close(gm, tot.cpu().numpy(), dt, f"case{ci}/call{call}/grad_mix")
                sums.append(gm.clone())
                calls.append((tg, th, tk, tm, ws, ref[2], gm_loc))
            # deferred form on the same inputs (the counter continues on the same buffers)
            prev = None
            for call, (tg, th, tk, tm, ws, own_ref, gm_loc) in enumerate(calls):
                gh, gk, gm = (torch.full_like(x, float("nan")) for x in (th, tk, tm))
                gprev = torch.full_like(tm, float("nan"))
                xch.backward_deferred(tg, th, tk, tm, gh, gk, gm, gprev, ws, off, dil)
                torch.cuda.synchronize()
                assert capi.device_error() == 0, capi.device_error_info()
                if dt != "fp32":  # same fixed-order local sum as the plain backward
                    assert torch.equal(gm, own_ref), (ci, call)
                assert_close(gm, gm_loc, dt, f"case{ci}/deferred{call}/own")
                if call == 0:
                    # the previous call on these buffers is the last synchronous one
                    assert torch.equal(gprev, sums[-1]), (ci, call)
                else:
                    assert torch.equal(gprev, sums[call - 1]), (ci, call)
            gfin = torch.full_like(calls[0][3], float("nan"))
            xch.finish(gfin)
            torch.cuda.synchronize()
            assert capi.device_error() == 0, capi.device_error_info()
            assert torch.equal(gfin, sums[-1]), ci
            dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException as e:  # noqa: BLE001  (reported to the parent)
        import traceback
        q.put((rank, "".join(traceback.format_exception(e))))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs (one rank per GPU)")
def test_dp_backward_exchange_ranks():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = min(torch.cuda.device_count(), 4)
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + 240
    while len(results) < world and time.time() < deadline:
        try:
            r, msg = q.get(timeout=5)
            results[r] = msg
        except Exception:  # noqa: BLE001
            if not all(p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert len(results) == world, f"ranks did not report: {results}"
    for r, msg in sorted(results.items()):
        assert msg == "ok", f"rank {r}:\n{msg}"
