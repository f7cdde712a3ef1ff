"""The Python API mirrors the reference's cuda_ops package: same names, module layout,
parameter shapes, and the same RuntimeError messages for bad inputs (checked here on
CPU tensors, where the reference raises before any launch)."""

import sys

import pytest
import torch

REF_EXPORTS = [
    "fused_dynamic_conv_chunk", "fused_dynamic_conv",
    "fused_dynamic_conv_forward_warmup_chunk", "fused_dynamic_conv_forward_warmup",
    "fused_dynamic_conv_forward_cached_plan_chunk", "fused_dynamic_conv_forward_cached_plan",
    "fused_dynamic_conv_forward_clear_warmup_cache", "fused_dynamic_conv_forward_plan_name",
    "fused_dynamic_conv_backward_warmup_chunk", "fused_dynamic_conv_backward_warmup",
    "fused_dynamic_conv_backward_cached_plan_chunk", "fused_dynamic_conv_backward_cached_plan",
    "fused_dynamic_conv_backward_clear_warmup_cache", "fused_dynamic_conv_backward_plan_name",
    "FusedDynamicConvChunkFunction", "FusedDynamicConvFunction", "FusedDynamicConvChunk1d",
    "FusedDynamicConv1d",
]
FSCM_EXPORTS = [
    "FORWARD_PLAN_GENERIC", "FORWARD_PLAN_C8S3", "FORWARD_PLAN_C32S3", "FORWARD_PLAN_D256C16S3",
    "FORWARD_PLAN_GENERIC_NO_BOUNDARY", "FORWARD_PLAN_C8S3_NO_BOUNDARY",
    "FORWARD_PLAN_C32S3_NO_BOUNDARY", "FORWARD_PLAN_D256C16S3_NO_BOUNDARY",
    "BACKWARD_PLAN_ATOMIC", "BACKWARD_PLAN_PER_D_REDUCE", "BACKWARD_PLAN_GATHER_X",
    "fused_source_conv_mixed", "fused_source_conv_mixed_forward",
    "fused_source_conv_mixed_forward_plan", "fused_source_conv_mixed_forward_cached_plan",
    "fused_source_conv_mixed_forward_warmup", "fused_source_conv_mixed_backward",
    "fused_source_conv_mixed_backward_plan", "fused_source_conv_mixed_backward_cached_plan",
    "fused_source_conv_mixed_backward_warmup", "fused_source_conv_mixed_backward_pack_cached_plan",
    "fused_source_conv_mixed_backward_cached_plan_get_plan",
    "fused_source_conv_mixed_backward_cached_plan_get_tile_t",
    "fused_source_conv_mixed_forward_plan_name", "fused_source_conv_mixed_backward_plan_name",
    "FusedSourceConvMixedFunction", "FusedSourceConvMixedChunk1d", "FusedSourceConvMixed1d",
]
EXT_FUNCS = ["forward_chunk", "forward_chunk_warmup", "forward_chunk_cached_plan",
             "forward_chunk_clear_warmup_cache", "forward_plan_name", "backward_chunk",
             "backward_chunk_warmup", "backward_chunk_cached_plan",
             "backward_chunk_clear_warmup_cache", "backward_plan_name"]
FSCM_OPS = ["forward", "forward_plan", "forward_cached_plan", "forward_warmup", "backward",
            "backward_plan", "backward_cached_plan", "backward_warmup",
            "backward_pack_cached_plan", "backward_cached_plan_get_plan",
            "backward_cached_plan_get_tile_t", "backward_atomic", "backward_per_d_reduce",
            "backward_gather_x"]


def test_api_surface():
    import dudyconv_b200.cuda_ops as co
    from dudyconv_b200.cuda_ops import fused_source_conv_mixed as fscm
    assert sorted(co.__all__) == sorted(REF_EXPORTS)
    for n in REF_EXPORTS:
        assert hasattr(co, n), n
    for n in FSCM_EXPORTS:
        assert hasattr(fscm, n), n
    ext = sys.modules["cuda_ops_ext"]
    for n in EXT_FUNCS:
        assert hasattr(ext, n), n
    for n in FSCM_OPS:
        assert hasattr(torch.ops.fused_source_conv_mixed, n), n
    assert fscm.FORWARD_PLAN_D256C16S3_NO_BOUNDARY == 103
    assert fscm.fused_source_conv_mixed_forward_plan_name(101) == "C8S3NoBoundary"
    assert fscm.fused_source_conv_mixed_backward_plan_name(2) == "GatherX"
    assert fscm.fused_source_conv_mixed_backward_plan_name(9) == "unknown_backward_plan_9"


def test_install_as_cuda_ops():
    import dudyconv_b200
    dudyconv_b200.install_as_cuda_ops()
    import cuda_ops  # noqa: F401
    from cuda_ops import fused_dynamic_conv_chunk
    from cuda_ops.fused_source_conv_mixed import fused_source_conv_mixed  # noqa: F401
    import dudyconv_b200.cuda_ops as co
    assert fused_dynamic_conv_chunk is co.fused_dynamic_conv_chunk


def test_cached_plan_packing():
    from dudyconv_b200.cuda_ops import fused_source_conv_mixed as fscm
    p = fscm.fused_source_conv_mixed_backward_pack_cached_plan(2, 128)
    assert fscm.fused_source_conv_mixed_backward_cached_plan_get_plan(p) == 2
    assert fscm.fused_source_conv_mixed_backward_cached_plan_get_tile_t(p) == 128
    assert p == 2 | (128 << 32)


def _t(*shape):
    return torch.zeros(*shape)


@pytest.mark.parametrize("args,msg", [
    ((_t(1, 4, 8), _t(1, 3, 2, 8), _t(4, 2), 0, 1), "h_full must be CUDA tensor."),
])
def test_forward_checks_cpu_tensors(args, msg):
    from dudyconv_b200.cuda_ops import fused_dynamic_conv_chunk
    with pytest.raises(RuntimeError, match=msg.replace(".", r"\.")):
        fused_dynamic_conv_chunk(*args)


def test_forward_checks_messages():
    from dudyconv_b200.cuda_ops.fused_dynamic_conv import _check_forward_inputs

    class FakeCuda:
        """Stand-in with .is_cuda so the shape checks run without a GPU."""

        def __init__(self, *shape, dtype=torch.float16):
            self.shape = torch.Size(shape)
            self.dtype = dtype
            self.is_cuda = True

        def dim(self):
            return len(self.shape)

    h, kc, mix = FakeCuda(1, 4, 8), FakeCuda(1, 3, 2, 8), FakeCuda(4, 2)
    _check_forward_inputs(h, kc, mix, 0, 1)
    cases = [
        ((h, kc, mix, 0, 0), "dilation must be positive."),
        ((FakeCuda(4, 8), kc, mix, 0, 1), "h_full must be [B,D,L], got (4, 8)."),
        ((h, FakeCuda(1, 3, 8), mix, 0, 1), "kernel_chunk must be [B,K,N,T], got (1, 3, 8)."),
        ((h, FakeCuda(2, 3, 2, 8), mix, 0, 1), "B mismatch: h_full=1, kernel_chunk=2."),
        ((h, kc, FakeCuda(5, 2), 0, 1), "D mismatch: h_full=4, kernel_mix=5."),
        ((h, kc, FakeCuda(4, 3), 0, 1), "N mismatch: kernel_chunk=2, kernel_mix=3."),
        ((h, kc, mix, -1, 1), "t_offset must be non-negative."),
        ((h, kc, mix, 1, 1), "t_offset + T must be <= L, got t_offset=1, T=8, L=8."),
        ((h, FakeCuda(1, 3, 2, 8, dtype=torch.float32), mix, 0, 1),
         "kernel_chunk dtype must equal h_full dtype."),
        ((FakeCuda(1, 4, 8, dtype=torch.int32), kc, mix, 0, 1), "Unsupported dtype: torch.int32."),
    ]
    for args, msg in cases:
        with pytest.raises(RuntimeError) as ei:
            _check_forward_inputs(*args)
        assert str(ei.value) == msg


def test_modules_construct():
    from dudyconv_b200.cuda_ops import FusedDynamicConv1d, FusedDynamicConvChunk1d
    from dudyconv_b200.cuda_ops.fused_source_conv_mixed import FusedSourceConvMixedChunk1d
    torch.manual_seed(0)
    m = FusedDynamicConvChunk1d(256, 128, use_bias=True)
    assert m.kernel_mix.shape == (256, 128) and m.bias.shape == (256,)
    assert abs(float(m.kernel_mix.std()) - 0.02) < 0.002
    assert FusedDynamicConv1d(8, 4).bias is None
    with pytest.raises(ValueError):
        FusedDynamicConvChunk1d(0, 4)
    s = FusedSourceConvMixedChunk1d(64, 16, 3)
    assert s.weight.shape == (64, 16, 3) and s.bias.shape == (64, 16)
    assert s.mix_weight.shape == (64, 16) and s.mix_bias.shape == (64,)
    assert FusedSourceConvMixedChunk1d(64, 16, 3, use_bias=False).bias is None
