"""Generate the golden fixtures under tests/golden/ from the REFERENCE's own formulas.

Run in the build container, where the reference checkout is readable:

    python tests/golden/make_golden.py --reference /path/to/DUDyConv

It imports the reference test modules (with a stub for the compiled
``cuda_ops_ext``, which the formulas do not use), evaluates

* ``torch_reference_materialized_chunk``
  (``test_fused_dynamic_conv_against_reference.py:91-189``) and
* ``torch_reference_source_conv_mixed_chunk``
  (``test_fused_source_conv_mixed.py:111-255``) and
* the kernel generator's ``StreamingKernelGenConv1d._logits_to_kernel``
  (``backbone_dil_unshared.py:1821-1900``)

in float64 on CPU, takes the backward with ``torch.autograd``, and writes the
outputs of every case to a compressed ``.npz``. Inputs are not stored: they are
re-drawn from the case seed by ``inputs.py`` (numpy PCG64, rounded to the
case dtype), which the tests call too. Outputs are stored as float32 (rounded
from float64).

The GPU box never runs this script: the fixtures travel with the repository.
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from inputs import fdc_inputs, fscm_inputs, kgen_inputs  # noqa: E402

# (name, B, D, L, T, N, K, off, dil, dtype, dist)
# "ref" distribution: randn * 0.1 for every tensor (the reference tests,
# test_fused_dynamic_conv_against_reference.py:41-68,380-417).
# "base" distribution: h, go ~ N(0,1); kc ~ N(0,1/N); mix ~ N(0,1/3).
FDC_CASES = [
    # reference quick cases (test_...:935-970)
    ("tiny_k1", 1, 1, 8, 8, 1, 1, 0, 1, "fp32", "ref"),
    ("small_offset0", 1, 16, 64, 32, 6, 3, 0, 1, "fp32", "ref"),
    ("odd_dilation2", 1, 17, 67, 19, 5, 4, 23, 2, "fp32", "ref"),
    # reference full cases (test_...:973-1095)
    ("B2_D31_dil4", 1, 31, 129, 64, 6, 3, 65, 4, "fp32", "ref"),
    ("D33_K5_dil8", 1, 33, 256, 113, 7, 5, 143, 8, "fp32", "ref"),
    ("full_len_dil16", 1, 64, 257, 257, 6, 3, 0, 16, "fp16", "ref"),
    ("near_tail", 1, 64, 511, 127, 8, 7, 384, 3, "fp16", "ref"),
    ("N1_K3", 1, 128, 512, 256, 1, 3, 128, 1, "bf16", "ref"),
    ("N2_K15_dil2", 1, 64, 1024, 256, 2, 15, 512, 2, "fp32", "ref"),
    ("N16_K3", 1, 128, 1024, 512, 16, 3, 256, 1, "fp16", "ref"),
    ("N32_K2", 1, 64, 1024, 512, 32, 2, 256, 1, "bf16", "ref"),
    # gradcheck shape (test_...:784-873) and full-length equivalence (test_...:599-780)
    ("gradcheck_shape", 1, 3, 7, 5, 2, 3, 1, 2, "fp32", "ref"),
    ("full_length_equiv", 1, 17, 65, 65, 5, 4, 0, 2, "fp32", "ref"),
    # hot-path shapes (D=256, K=3, N in {16..128}) at reduced B and T
    ("hot_n16_d256", 1, 256, 128, 128, 16, 3, 0, 1, "fp16", "base"),
    ("hot_n32_d256_b2", 2, 256, 64, 64, 32, 3, 0, 1, "fp16", "base"),
    ("hot_n64_d256_bf16", 1, 256, 128, 128, 64, 3, 0, 1, "bf16", "base"),
    ("hot_n128_d256", 1, 256, 64, 64, 128, 3, 0, 1, "fp16", "base"),
    ("hot_n128_chunk_off", 1, 256, 192, 64, 128, 3, 128, 1, "fp16", "base"),
    ("hot_n32_dil32", 1, 256, 192, 192, 32, 3, 0, 32, "fp16", "base"),
    ("hot_n64_ragged_t72", 1, 128, 96, 72, 64, 3, 16, 2, "fp16", "base"),
    ("hot_n16_fp32", 1, 256, 128, 128, 16, 3, 0, 1, "fp32", "base"),
]

# (name, B, D, L, T, C, S, off, dil, use_bias, dtype)
# all randn * 0.1 (test_fused_source_conv_mixed.py:380-417 uses the same scale)
FSCM_CASES = [
    ("tiny_c1_s1_bias", 1, 1, 8, 8, 1, 1, 0, 1, True, "fp32"),
    ("tiny_c1_s1_nobias", 1, 2, 8, 8, 1, 1, 0, 1, False, "fp32"),
    ("boundary_c8_s3", 1, 16, 64, 32, 8, 3, 0, 1, True, "fp32"),
    ("noboundary_c8_s3", 1, 16, 64, 32, 8, 3, 8, 1, True, "fp16"),
    ("odd_dilation2_c5_s4", 1, 17, 67, 19, 5, 4, 23, 2, True, "fp32"),
    ("c32_s3_boundary", 1, 64, 96, 64, 32, 3, 0, 1, True, "fp16"),
    ("c32_s3_noboundary", 1, 64, 128, 64, 32, 3, 16, 1, False, "bf16"),
    ("d256_c16_s3_dil4", 1, 256, 256, 64, 16, 3, 128, 4, True, "fp16"),
    ("batch2_d64_c8_s3", 2, 64, 256, 128, 8, 3, 64, 1, True, "fp32"),
    ("generic_c7_s5", 1, 33, 257, 113, 7, 5, 143, 3, True, "fp32"),
    ("c16_s8", 1, 128, 512, 128, 16, 8, 128, 2, False, "fp16"),
    ("hot_d256_c16_s3_dil16", 1, 256, 128, 128, 16, 3, 0, 16, True, "fp16"),
    ("hot_d256_c3_s3_dil1", 2, 256, 64, 64, 3, 3, 0, 1, True, "bf16"),
]


# (name, B, N, K, T, dtype): the kernel generator's tail, StreamingKernelGenConv1d.
# _logits_to_kernel (backbone_dil_unshared.py:1821-1900); logits ~ N(0, 1.5^2)
KGEN_CASES = [
    ("n128_k3_t64", 2, 128, 3, 64, "fp16"),
    ("n16_k3_t40", 1, 16, 3, 40, "fp32"),
    ("n8_k5_t33", 2, 8, 5, 33, "bf16"),
    ("n4_k1_t16", 1, 4, 1, 16, "fp32"),
    ("n6_k20_t24", 1, 6, 20, 24, "fp16"),
]


def _import_reference(ref_dir: str):
    sys.modules.setdefault("cuda_ops_ext", types.ModuleType("cuda_ops_ext"))
    sys.path.insert(0, ref_dir)
    import test_fused_dynamic_conv_against_reference as fdc_ref  # noqa: E402
    import test_fused_source_conv_mixed as fscm_ref  # noqa: E402
    return fdc_ref, fscm_ref


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).double()


def make_fdc(fdc_ref, idx, case):
    name, B, D, L, T, N, K, off, dil, dtype, dist = case
    meta = np.array([B, D, L, T, N, K, off, dil], dtype=np.int64)
    seed = 1234 + idx
    h, kc, mix, go = fdc_inputs(meta, dtype, dist, seed)
    hd, kd, md = (_t(a).requires_grad_(True) for a in (h, kc, mix))
    out = fdc_ref.torch_reference_materialized_chunk(hd, kd, md, t_offset=off, dilation=dil)
    out.backward(_t(go))
    # cross-check with the reference's second formula (test_...:191-282)
    out2 = fdc_ref.torch_reference_no_materialize_chunk(
        _t(h), _t(kc), _t(mix), t_offset=off, dilation=dil)
    assert torch.allclose(out, out2, rtol=1e-12, atol=1e-12), name
    return {
        "meta": meta, "dtype": np.array(dtype), "dist": np.array(dist),
        "seed": np.array(seed, dtype=np.int64),
        "out": out.detach().float().numpy(),
        "grad_h": hd.grad.float().numpy(),
        "grad_kc": kd.grad.float().numpy(),
        "grad_mix": md.grad.float().numpy(),
    }


def make_fscm(fscm_ref, idx, case):
    name, B, D, L, T, C, S, off, dil, use_bias, dtype = case
    meta = np.array([B, D, L, T, C, S, off, dil, int(use_bias)], dtype=np.int64)
    seed = 4321 + idx
    x, w, bias, mw, mb, go = fscm_inputs(meta, dtype, seed)
    xd, wd, mwd, mbd = (_t(a).requires_grad_(True) for a in (x, w, mw, mb))
    bd = _t(bias).requires_grad_(True) if use_bias else None
    out = fscm_ref.torch_reference_source_conv_mixed_chunk(xd, wd, bd, mwd, mbd, off, T, dil)
    out.backward(_t(go))
    rec = {
        "meta": meta, "dtype": np.array(dtype), "seed": np.array(seed, dtype=np.int64),
        "out": out.detach().float().numpy(),
        "grad_x": xd.grad.float().numpy(),
        "grad_w": wd.grad.float().numpy(),
        "grad_mix_w": mwd.grad.float().numpy(),
        "grad_mix_b": mbd.grad.float().numpy(),
    }
    if use_bias:
        rec["grad_bias"] = bd.grad.float().numpy()
    return rec


def make_kgen(idx, case):
    """Forward and autograd backward of the reference model's own _logits_to_kernel."""
    import backbone_dil_unshared as bb  # noqa: E402  (imported after _import_reference)

    name, B, N, K, T, dtype = case
    meta = np.array([B, N, K, T], dtype=np.int64)
    seed = 777 + idx
    logits, gkc = kgen_inputs(meta, dtype, seed)
    gen = bb.StreamingKernelGenConv1d(embed_dim=4, num_kernels=N, dynamic_kernel_size=K,
                                      kernel_gen_kernel_size=3, bias=True).double()
    ld = _t(logits).requires_grad_(True)
    kc = gen._logits_to_kernel(ld, T)
    kc.backward(_t(gkc))
    return {"meta": meta, "dtype": np.array(dtype), "seed": np.array(seed, dtype=np.int64),
            "kc": kc.detach().float().numpy(), "grad_logits": ld.grad.float().numpy()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the DUDyConv checkout")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    fdc_ref, fscm_ref = _import_reference(args.reference)
    fdc = {}
    for i, case in enumerate(FDC_CASES):
        for k, v in make_fdc(fdc_ref, i, case).items():
            fdc[f"{case[0]}/{k}"] = v
    np.savez_compressed(os.path.join(args.out, "fdc_golden.npz"), **fdc)
    fscm = {}
    for i, case in enumerate(FSCM_CASES):
        for k, v in make_fscm(fscm_ref, i, case).items():
            fscm[f"{case[0]}/{k}"] = v
    np.savez_compressed(os.path.join(args.out, "fscm_golden.npz"), **fscm)
    kgen = {}
    for i, case in enumerate(KGEN_CASES):
        for k, v in make_kgen(i, case).items():
            kgen[f"{case[0]}/{k}"] = v
    np.savez_compressed(os.path.join(args.out, "kgen_golden.npz"), **kgen)
    print("wrote", len(FDC_CASES), "fdc cases,", len(FSCM_CASES), "fscm cases and",
          len(KGEN_CASES), "kernel-generator cases")


if __name__ == "__main__":
    main()
