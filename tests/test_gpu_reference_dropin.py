"""The reference's own, unchanged Python code running on this library's kernels.

The reference's ``cuda_ops/*.py`` (its autograd Functions, wrappers and warmup helpers),
its two test modules and its model file are imported from a staged copy of the reference
(``baseline/_ref/``, made by ``tests/stage_reference.py``; or the directory named by
``DUDY_REFERENCE_DIR``), with this library's compiled binding registered under the name
they import, ``cuda_ops_ext``. Nothing of the reference is edited: its Python layer calls
``cuda_ops_ext.forward_chunk`` / ``backward_chunk`` / ``*_warmup`` / ``*_cached_plan`` and
``torch.ops.fused_source_conv_mixed.*`` exactly as it would call its own extension.

* The reference's correctness bodies for its ``--quick`` and ``--full`` case lists, in
  fp32 / fp16 / bf16, with the seeds its CLI uses (``1234 + case index``):
  ``test_fused_dynamic_conv_against_reference.py:369-589`` (warmup -> cached-plan
  equality asserts, forward, backward, against its own PyTorch formulas and
  tolerances) and ``test_fused_source_conv_mixed.py:804-1160`` (every legal forward plan,
  every backward (plan, tile_t) pair), plus its full-length equivalence and cached-plan
  bodies.
* One ``DilatedUnsharedLayer`` (``backbone_dil_unshared.py:3571``; D=256, N=128, K=3,
  C=16, chunk 256, so the op runs per 256-token chunk with ``t_offset``) forward and
  backward with ``dynamic_conv_impl="cuda_fused"``, against the same layer (same weights,
  same code path) with ``cuda_ops.fused_dynamic_conv_chunk`` replaced by the reference's
  own PyTorch formula (``torch_reference_materialized_chunk``,
  ``test_fused_dynamic_conv_against_reference.py:91-189``), comparing outputs and every
  parameter gradient. (The model's other PyTorch paths, e.g.
  ``materialized_kernel_stream_x``, apply ``norm1`` to the window themselves
  (``backbone_dil_unshared.py:2748-2800``) while the fused path passes ``h_full`` as is,
  so they are not the same function as the fused path.)

The module skips, with the reason, when no staged reference is present.
"""

from __future__ import annotations

import importlib
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.environ.get("DUDY_REFERENCE_DIR") or os.path.join(ROOT, "baseline", "_ref")
HAVE_REF = os.path.exists(os.path.join(REF_DIR, "backbone_dil_unshared.py")) and \
    os.path.exists(os.path.join(REF_DIR, "cuda_ops", "fused_dynamic_conv.py"))

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not HAVE_REF, reason=f"no staged reference checkout at {REF_DIR} "
                       "(run `python tests/stage_reference.py <checkout>`)"),
]

_REF_MODULES = ("test_fused_dynamic_conv_against_reference", "test_fused_source_conv_mixed",
                "backbone_dil_unshared")


def _is_ops(name: str) -> bool:
    return name in ("cuda_ops", "cuda_ops_ext") or name.startswith("cuda_ops.")


@pytest.fixture(scope="module")
def ref():
    """Import the reference's modules over this library's binding; restore on exit."""
    import dudyconv_b200

    saved = {k: v for k, v in sys.modules.items() if _is_ops(k) or k in _REF_MODULES}
    for k in saved:
        del sys.modules[k]
    sys.modules["cuda_ops_ext"] = dudyconv_b200.load_extension()
    sys.path.insert(0, REF_DIR)
    try:
        ops = importlib.import_module("cuda_ops")
        assert os.path.dirname(os.path.abspath(ops.__file__)) == \
            os.path.join(os.path.abspath(REF_DIR), "cuda_ops"), ops.__file__
        mods = {m: importlib.import_module(m) for m in _REF_MODULES}
        yield mods
    finally:
        sys.path.remove(REF_DIR)
        for k in [k for k in sys.modules if _is_ops(k) or k in _REF_MODULES]:
            del sys.modules[k]
        sys.modules.update(saved)


DTYPES = [torch.float32, torch.float16, torch.bfloat16]
DT_IDS = ["fp32", "fp16", "bf16"]


@pytest.mark.parametrize("dtype", DTYPES, ids=DT_IDS)
@pytest.mark.parametrize("suite", ["quick", "full"])
def test_reference_dynamic_conv_cases(ref, suite, dtype):
    t = ref["test_fused_dynamic_conv_against_reference"]
    cases = t.get_quick_cases() if suite == "quick" else t.get_full_cases()
    for idx, case in enumerate(cases):
        t.run_correctness_case_body(case, dtype, seed=1234 + idx)


@pytest.mark.parametrize("dtype", DTYPES, ids=DT_IDS)
def test_reference_dynamic_conv_full_length(ref, dtype):
    ref["test_fused_dynamic_conv_against_reference"].run_full_length_equivalence_body(dtype)


@pytest.mark.parametrize("dtype", DTYPES, ids=DT_IDS)
@pytest.mark.parametrize("suite", ["quick", "full"])
def test_reference_source_conv_cases(ref, suite, dtype):
    t = ref["test_fused_source_conv_mixed"]
    cases = t.get_quick_cases() if suite == "quick" else t.get_full_cases()
    for idx, case in enumerate(cases):
        t.run_correctness_case_body(case, dtype, seed=1234 + idx)


@pytest.mark.parametrize("dtype", DTYPES, ids=DT_IDS)
def test_reference_source_conv_cached_plan_api(ref, dtype):
    ref["test_fused_source_conv_mixed"].run_cached_plan_body(dtype)


def _layer(bb, dilation):
    torch.manual_seed(0)
    return bb.DilatedUnsharedLayer(
        embed_dim=256, source_channels=16, num_kernels=128, dynamic_kernel_size=3,
        source_conv_kernel_size=3, kernel_gen_kernel_size=3, dilation=dilation,
        mlp_ratio=4.0, dropout=0.0, normalize_kernel=True, initial_scale=0.1,
        use_bias=True, use_checkpoint=False, dynamic_conv_impl="cuda_fused",
        use_nonlinear_residual=True, nonlinear_residual_initial_scale=0.05)


def _run_layer(layer, src, dyn, chunk, op=None):
    """Forward + backward of the layer; ``op`` replaces cuda_ops.fused_dynamic_conv_chunk
    (the name the layer imports at call time) for this run."""
    ops = sys.modules["cuda_ops"]
    saved = ops.fused_dynamic_conv_chunk
    if op is not None:
        ops.fused_dynamic_conv_chunk = op
    try:
        src = src.detach().clone().requires_grad_(True)
        dyn = dyn.detach().clone().requires_grad_(True)
        a, b = layer(src, dyn, chunk_size=chunk)
        g = torch.Generator(device=src.device).manual_seed(1)
        wa = torch.randn(a.shape, device=src.device, generator=g, dtype=torch.float32)
        wb = torch.randn(b.shape, device=src.device, generator=g, dtype=torch.float32)
        loss = (a.float() * wa).sum() + (b.float() * wb).sum()
        loss.backward()
    finally:
        ops.fused_dynamic_conv_chunk = saved
    res = {"next_source": a.detach(), "next_dynamic": b.detach(), "grad_src": src.grad,
           "grad_dyn": dyn.grad}
    for name, p in layer.named_parameters():
        res["grad/" + name] = p.grad
    return res


def _max_rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.mark.parametrize("dilation", [2, 16])
def test_backbone_layer_on_the_op(ref, dilation):
    """A DilatedUnsharedLayer whose dynamic conv runs through this library (per 256-token
    chunk, with the layer's warmup) against the same layer running the reference's own
    PyTorch formula for the op."""
    bb = ref["backbone_dil_unshared"]
    formula = ref["test_fused_dynamic_conv_against_reference"].torch_reference_materialized_chunk
    B, D, L, chunk = 2, 256, 1024, 256
    g = torch.Generator(device="cuda").manual_seed(5)
    src = torch.randn(B, D, L, device="cuda", generator=g)
    dyn = torch.randn(B, D, L, device="cuda", generator=g)

    # float64, reference formula: the accuracy reference
    exact = _run_layer(_layer(bb, dilation).cuda().double(), src.double(), dyn.double(), chunk,
                       op=formula)
    # fp32: this library's op (CUDA-core plan) against the formula, both in fp32
    ours32 = _run_layer(_layer(bb, dilation).cuda(), src, dyn, chunk)
    theirs32 = _run_layer(_layer(bb, dilation).cuda(), src, dyn, chunk, op=formula)
    assert ours32.keys() == exact.keys()
    # parameters the fused path does not use (its norm1: the op gets h_full as is) have no
    # gradient on either side
    unused = {k for k in exact if exact[k] is None}
    assert all(k.startswith("grad/") for k in unused), unused
    assert len(unused) < len(exact) // 4, unused
    for k in exact:
        if k in unused:
            assert ours32[k] is None and theirs32[k] is None, k
            continue
        assert ours32[k] is not None, k
        assert _max_rel(ours32[k], theirs32[k]) < 1e-4, (k, _max_rel(ours32[k], theirs32[k]))
    # fp16 (tensor-core plan, after the layer's own warmup): at least as close to the
    # float64 result as the reference formula evaluated in fp16 (plus a small margin)
    layer16 = _layer(bb, dilation).cuda().half()
    layer16.warmup_cuda_dynamic_conv(batch_size=B, seq_len=L, chunk_size=chunk,
                                     device=torch.device("cuda"), dtype=torch.float16,
                                     repeat=1)
    ours16 = _run_layer(layer16, src.half(), dyn.half(), chunk)
    theirs16 = _run_layer(_layer(bb, dilation).cuda().half(), src.half(), dyn.half(), chunk,
                          op=formula)
    for k in exact:
        if k in unused:
            continue
        e_ours, e_theirs = _max_rel(ours16[k], exact[k]), _max_rel(theirs16[k], exact[k])
        assert e_ours <= 1.5 * e_theirs + 2e-3, (k, e_ours, e_theirs)


@pytest.mark.parametrize("dilation", [2, 16])
def test_backbone_layer_with_fused_source_conv_and_kernel_tail(ref, dilation):
    """dudyconv_b200.backbone.install routes the layer's source path
    (forward_mixed_chunk, backbone_dil_unshared.py:1263-1512) to fused_source_conv_mixed and
    the kernel generator's softmax + flip (:1821-1900) to the fused logits_to_kernel; the
    layer's outputs and every gradient must match the unpatched layer."""
    from dudyconv_b200.backbone import install

    bb = ref["backbone_dil_unshared"]
    formula = ref["test_fused_dynamic_conv_against_reference"].torch_reference_materialized_chunk
    B, D, L, chunk = 2, 256, 1024, 256
    g = torch.Generator(device="cuda").manual_seed(9)
    src = torch.randn(B, D, L, device="cuda", generator=g)
    dyn = torch.randn(B, D, L, device="cuda", generator=g)
    # the reference layer, all PyTorch (its einsum source path, its softmax, the op's
    # formula), in float64: the accuracy reference
    exact = _run_layer(_layer(bb, dilation).cuda().double(), src.double(), dyn.double(), chunk,
                       op=formula)
    plain32 = _run_layer(_layer(bb, dilation).cuda(), src, dyn, chunk)
    plain16 = _run_layer(_layer(bb, dilation).cuda().half(), src.half(), dyn.half(), chunk,
                         op=formula)
    restore = install(bb)
    try:
        fused32 = _run_layer(_layer(bb, dilation).cuda(), src, dyn, chunk)
        fused16 = _run_layer(_layer(bb, dilation).cuda().half(), src.half(), dyn.half(), chunk)
    finally:
        restore()
    for k in exact:
        if exact[k] is None:
            assert fused32[k] is None, k
            continue
        assert _max_rel(fused32[k], plain32[k]) < 1e-4, (k, _max_rel(fused32[k], plain32[k]))
        e_ours, e_theirs = _max_rel(fused16[k], exact[k]), _max_rel(plain16[k], exact[k])
        assert e_ours <= 1.5 * e_theirs + 2e-3, (k, e_ours, e_theirs)
