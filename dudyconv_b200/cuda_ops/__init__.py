"""Drop-in replacement of the reference's ``cuda_ops`` package (same 18 exports;
``fused_source_conv_mixed`` is a submodule, as in the reference's
``cuda_ops/__init__.py``)."""

from .fused_dynamic_conv import (  # noqa: F401
    FusedDynamicConv1d,
    FusedDynamicConvChunk1d,
    FusedDynamicConvChunkFunction,
    FusedDynamicConvFunction,
    fused_dynamic_conv,
    fused_dynamic_conv_backward_cached_plan,
    fused_dynamic_conv_backward_cached_plan_chunk,
    fused_dynamic_conv_backward_clear_warmup_cache,
    fused_dynamic_conv_backward_plan_name,
    fused_dynamic_conv_backward_warmup,
    fused_dynamic_conv_backward_warmup_chunk,
    fused_dynamic_conv_chunk,
    fused_dynamic_conv_forward_cached_plan,
    fused_dynamic_conv_forward_cached_plan_chunk,
    fused_dynamic_conv_forward_clear_warmup_cache,
    fused_dynamic_conv_forward_plan_name,
    fused_dynamic_conv_forward_warmup,
    fused_dynamic_conv_forward_warmup_chunk,
)

__all__ = [
    "fused_dynamic_conv_chunk",
    "fused_dynamic_conv",
    "fused_dynamic_conv_forward_warmup_chunk",
    "fused_dynamic_conv_forward_warmup",
    "fused_dynamic_conv_forward_cached_plan_chunk",
    "fused_dynamic_conv_forward_cached_plan",
    "fused_dynamic_conv_forward_clear_warmup_cache",
    "fused_dynamic_conv_forward_plan_name",
    "fused_dynamic_conv_backward_warmup_chunk",
    "fused_dynamic_conv_backward_warmup",
    "fused_dynamic_conv_backward_cached_plan_chunk",
    "fused_dynamic_conv_backward_cached_plan",
    "fused_dynamic_conv_backward_clear_warmup_cache",
    "fused_dynamic_conv_backward_plan_name",
    "FusedDynamicConvChunkFunction",
    "FusedDynamicConvFunction",
    "FusedDynamicConvChunk1d",
    "FusedDynamicConv1d",
]
