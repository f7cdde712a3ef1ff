"""Data-parallel host logic on CPU: two gloo ranks each take their shard of the batch,
compute their local gradients (float64 oracle, standing in for the device op), and the
grad_mix all-reduce must reproduce the full-batch gradient."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dudyconv_b200.dp import allreduce_grad_mix, shard_range


def test_shard_range_partitions():
    for B in (1, 5, 16, 17):
        for world in (1, 2, 3, 8):
            spans = [shard_range(B, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import fdc_backward

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.Generator(np.random.PCG64(7))
        B, D, L, T, N, K = 5, 16, 40, 40, 6, 3
        h = rng.standard_normal((B, D, L))
        kc = rng.standard_normal((B, K, N, T))
        mix = rng.standard_normal((D, N))
        go = rng.standard_normal((B, D, T))
        a, b = shard_range(B, rank, world)
        _, _, gm = fdc_backward(go[a:b], h[a:b], kc[a:b], mix, 0, 1)
        t = torch.from_numpy(gm.astype(np.float32)).to(torch.float16)
        allreduce_grad_mix(t)
        _, _, gm_full = fdc_backward(go, h, kc, mix, 0, 1)
        err = float(np.abs(t.float().numpy() - gm_full).max() / np.abs(gm_full).max())
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


def test_grad_mix_allreduce_matches_full_batch():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, err in res:
        assert err < 2e-3, (rank, err)  # fp16 storage of the reduced result


def _torch_chunk_op(h_full, kc, mix, t_offset, dil):
    """The op's formula in float64 torch (differentiable), standing in for the device op:
    out[b,d,t] = sum_k sum_n h_full[b,d, t_offset + t - k*dil] kc[b,k,n,t] mix[d,n] (zero
    before position 0)."""
    K, T = kc.shape[1], kc.shape[3]
    hp = torch.nn.functional.pad(h_full, ((K - 1) * dil, 0))
    out = 0
    for k in range(K):
        s = t_offset - k * dil + (K - 1) * dil
        out = out + torch.einsum("bnt,dn->bdt", kc[:, k], mix) * hp[..., s:s + T]
    return out


def _seq_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from dudyconv_b200.dp import sequence_sharded_dynamic_conv

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(11)
        B, D, N, K, dil, L = 2, 6, 4, 3, 2, 24
        h = torch.randn(B, D, L, generator=g, dtype=torch.float64)
        kc = torch.randn(B, K, N, L, generator=g, dtype=torch.float64)
        mix = torch.randn(D, N, generator=g, dtype=torch.float64)
        go = torch.randn(B, D, L, generator=g, dtype=torch.float64)
        # whole sequence on one rank
        hr, kr, mr = (t.clone().requires_grad_() for t in (h, kc, mix))
        out_ref = _torch_chunk_op(hr, kr, mr, 0, dil)
        (out_ref * go).sum().backward()
        # this rank's slice of the time axis
        Ls = L // world
        sl = slice(rank * Ls, (rank + 1) * Ls)
        hl = h[..., sl].clone().requires_grad_()
        kl = kc[..., sl].clone().requires_grad_()
        ml = mix.clone().requires_grad_()
        out = sequence_sharded_dynamic_conv(hl, kl, ml, dil, op=_torch_chunk_op)
        (out * go[..., sl]).sum().backward()
        gm = ml.grad.clone()
        dist.all_reduce(gm)
        errs = [float((out - out_ref[..., sl]).abs().max()),
                float((hl.grad - hr.grad[..., sl]).abs().max()),
                float((kl.grad - kr.grad[..., sl]).abs().max()),
                float((gm - mr.grad).abs().max())]
        q.put((rank, max(errs)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sequence_sharded_halo_exchange_matches_whole_sequence(world):
    """Sequence sharding across gloo ranks on CPU: outputs and every gradient of the sharded
    op (one causal halo exchange each way) equal those of the whole sequence on one rank."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_seq_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, err in res:
        assert err < 1e-10, (rank, err)
