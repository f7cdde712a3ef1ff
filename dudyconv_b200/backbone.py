"""Route the reference model's remaining PyTorch hot spots to this library, unchanged.

``backbone_dil_unshared.py`` (adjfangjiawei/DUDyConv) already calls the dynamic conv
through ``cuda_ops.fused_dynamic_conv_chunk``; ``dudyconv_b200.install_as_cuda_ops()``
makes that call land here. Two more per-chunk steps of every layer stay in PyTorch in
the reference, and ``install(backbone_module)`` routes them here too, without editing the
model file (the methods are replaced on the classes of the module object passed in):

* ``ChunkedDUnsharedDilatedSourceConv1d.forward_mixed_chunk``
  (``backbone_dil_unshared.py:1263-1512``): windows -> einsum -> GELU -> einsum per
  source-channel block, then ``+ source_mix_bias`` and the post-mix dropout. This is
  exactly ``fused_source_conv_mixed(x_full, weight, bias, mix_w, mix_b, off=start,
  T=end-start, dilation)`` (``cuda_ops/fused_source_conv_mixed.py:356``) followed by the
  dropout, when the activation is the exact (erf) GELU and the tensors are on a GPU.
* ``StreamingKernelGenConv1d._logits_to_kernel`` (``backbone_dil_unshared.py:1821-1900``):
  softmax over K, flip, permute, as the fused one-pass ``logits_to_kernel``.

Anything the fused ops do not cover (CPU tensors, another activation) keeps running the
model's own method. ``install`` returns a function that restores the original methods.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.nn as nn


def _fused_forward_mixed_chunk(orig):
    from .cuda_ops.fused_source_conv_mixed import fused_source_conv_mixed

    def forward_mixed_chunk(self, x_full, start, end, source_mix_weight, source_mix_bias,
                            activation, dropout_module, post_mix_dropout_module):
        exact_gelu = isinstance(activation, nn.GELU) and \
            getattr(activation, "approximate", "none") == "none"
        if not (torch.is_tensor(x_full) and x_full.is_cuda and exact_gelu and
                x_full.dim() == 3):
            return orig(self, x_full, start, end, source_mix_weight, source_mix_bias,
                        activation, dropout_module, post_mix_dropout_module)
        B, D, L = x_full.shape
        if D != self.embed_dim:
            raise ValueError(f"embed_dim mismatch: expected {self.embed_dim}, got {D}")
        start_i, end_i = int(start), int(end)
        if not (0 <= start_i < end_i <= L):
            raise ValueError(f"bad chunk bounds start={start_i}, end={end_i}, L={L}")
        dt = x_full.dtype
        # the op takes one dtype for all tensors (the model's dynamic-conv path casts its
        # parameters to the activation dtype the same way, backbone_dil_unshared.py:3036-3052)
        weight = self.weight.to(dt)
        bias = self.bias.to(dt) if self.bias is not None else None
        out = fused_source_conv_mixed(x_full.contiguous(), weight, bias,
                                      source_mix_weight.to(dt), source_mix_bias.to(dt),
                                      start_i, end_i - start_i, int(self.dilation))
        return post_mix_dropout_module(out)

    return forward_mixed_chunk


def _fused_logits_to_kernel(orig):
    from .kernel_gen import logits_to_kernel

    def _logits_to_kernel(self, logits, expected_T):
        if not (torch.is_tensor(logits) and logits.is_cuda and logits.dim() == 3):
            return orig(self, logits, expected_T)
        B, M, T = logits.shape
        if M != self.kernel_channels:
            raise ValueError(f"logits channels: expected {self.kernel_channels}, got {M}")
        if T != int(expected_T):
            raise RuntimeError(f"logits length: expected {int(expected_T)}, got {T}")
        return logits_to_kernel(logits, self.num_kernels, self.dynamic_kernel_size)

    return _logits_to_kernel


def install(backbone_module, source_conv: bool = True, kernel_tail: bool = True) -> Callable[[], None]:
    """Replace the two methods on the classes of ``backbone_module`` (the imported
    ``backbone_dil_unshared``); returns a function that puts the originals back."""
    undo = []
    if source_conv:
        cls = backbone_module.ChunkedDUnsharedDilatedSourceConv1d
        orig = cls.forward_mixed_chunk
        cls.forward_mixed_chunk = _fused_forward_mixed_chunk(orig)
        undo.append((cls, "forward_mixed_chunk", orig))
    if kernel_tail:
        cls = backbone_module.StreamingKernelGenConv1d
        orig = cls._logits_to_kernel
        cls._logits_to_kernel = _fused_logits_to_kernel(orig)
        undo.append((cls, "_logits_to_kernel", orig))

    def restore():
        for c, name, fn in reversed(undo):
            setattr(c, name, fn)

    return restore
