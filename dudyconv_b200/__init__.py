"""dudyconv_b200 -- B200 (sm_100a) fused dynamic causal convolution and fused source conv.

Drop-in for the ``cuda_ops`` package of adjfangjiawei/DUDyConv:

* ``dudyconv_b200.cuda_ops``  -- the same Python API (autograd Functions, functional
  wrappers, warmup / cached-plan helpers, ``nn.Module`` wrappers) as the reference's
  ``cuda_ops/fused_dynamic_conv.py`` and ``cuda_ops/fused_source_conv_mixed.py``.
* ``cuda_ops_ext``            -- the compiled torch binding (built in-tree by
  ``dudyconv_b200.build``) over the C ABI of ``libdudyconv_b200.so``.

``install_as_cuda_ops()`` registers both under the reference's import names
(``cuda_ops``, ``cuda_ops.fused_dynamic_conv``, ``cuda_ops.fused_source_conv_mixed``,
``cuda_ops_ext``) so unmodified callers such as ``backbone_dil_unshared.py`` use this
implementation.

There is no CPU or library fallback: if the native extension is missing, importing
``dudyconv_b200.cuda_ops`` raises ImportError.
"""

from __future__ import annotations

import importlib
import os
import sys

__version__ = "0.1.0"

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
_EXT = None


def load_extension():
    """Import the in-tree ``cuda_ops_ext`` module (raises ImportError if it is not built)."""
    global _EXT
    if _EXT is not None:
        return _EXT
    import torch  # noqa: F401  (loads libc10 / libtorch before the extension)

    try:
        _EXT = importlib.import_module("dudyconv_b200.cuda_ops_ext")
    except ImportError as e:
        raise ImportError(
            "dudyconv_b200: the native extension cuda_ops_ext is not built "
            f"({e}). Build it with `python -m dudyconv_b200.build`."
        ) from e
    sys.modules.setdefault("cuda_ops_ext", _EXT)
    return _EXT


def install_as_cuda_ops() -> None:
    """Make ``import cuda_ops`` / ``import cuda_ops_ext`` resolve to this package."""
    load_extension()
    from . import cuda_ops
    from .cuda_ops import fused_dynamic_conv, fused_source_conv_mixed

    sys.modules["cuda_ops"] = cuda_ops
    sys.modules["cuda_ops.fused_dynamic_conv"] = fused_dynamic_conv
    sys.modules["cuda_ops.fused_source_conv_mixed"] = fused_source_conv_mixed


def build_native() -> None:
    """Compile the native libraries in-tree (nvcc for sm_100a, g++ for the binding)."""
    from .build import build

    build()
