"""Sequence sharding on two GPUs (NCCL): each rank holds half of the time axis, exchanges the
causal halo with its neighbour, and runs the tensor-core op; outputs and gradients must match
the whole sequence computed on one GPU. Skipped with fewer than two GPUs."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.join(here, "golden"))
    import datetime

    import torch.distributed as dist

    from dudyconv_b200.cuda_ops import fused_dynamic_conv_chunk
    from dudyconv_b200.dp import allreduce_grad_mix, sequence_sharded_dynamic_conv
    from parity import assert_close

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        g = torch.Generator(device=dev).manual_seed(5)
        B, D, N, K, dil, L = 2, 256, 128, 3, 4, 2048
        h = torch.randn(B, D, L, device=dev, generator=g).half()
        kc = (torch.randn(B, K, N, L, device=dev, generator=g) * N ** -0.5).half()
        mix = (torch.randn(D, N, device=dev, generator=g) * 3 ** -0.5).half()
        go = torch.randn(B, D, L, device=dev, generator=g).half()
        hr, kr, mr = (t.clone().requires_grad_() for t in (h, kc, mix))
        out_ref = fused_dynamic_conv_chunk(hr, kr, mr, 0, dil)
        out_ref.backward(go)
        Ls = L // world
        sl = slice(rank * Ls, (rank + 1) * Ls)
        hl = h[..., sl].clone().requires_grad_()
        kl = kc[..., sl].clone().requires_grad_()
        ml = mix.clone().requires_grad_()
        out = sequence_sharded_dynamic_conv(hl, kl, ml, dil)
        out.backward(go[..., sl].contiguous())
        allreduce_grad_mix(ml.grad)
        torch.cuda.synchronize()

        def ref64(t):
            return t.detach().double().cpu().numpy()

        assert_close(out, ref64(out_ref[..., sl]), "fp16", "out")
        assert_close(hl.grad, ref64(hr.grad[..., sl]), "fp16", "grad_h")
        assert_close(kl.grad, ref64(kr.grad[..., sl]), "fp16", "grad_kc")
        # grad_mix: each rank's op call returns its partial sum rounded to fp16, and the ranks
        # add those (allreduce_grad_mix); the reference is that sum of the float64 partials,
        # each rounded to fp16 (the rounding of the partials is the exchange's, not the op's)
        from oracle.fdc_torch import fdc_backward_t
        H = (K - 1) * dil
        prev = h[..., rank * Ls - H: rank * Ls] if rank > 0 else torch.zeros_like(h[..., :H])
        h_ext = torch.cat([prev, h[..., sl]], dim=-1)
        part = fdc_backward_t(go[..., sl].contiguous(), h_ext, kc[..., sl].contiguous(), mix,
                              H, dil)[2].half().float()
        dist.all_reduce(part)
        assert_close(ml.grad, part.double().cpu().numpy(), "fp16", "grad_mix")
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)[:400]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sequence_sharded_two_gpus_matches_whole_sequence():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, msg in res:
        assert msg == "ok", (rank, msg)
