"""Stage the reference's Python sources for the drop-in tests.

    python tests/stage_reference.py <reference checkout> [<destination>]

Copies the reference's model, test and ``cuda_ops/*.py`` files, unchanged, from a
checkout of adjfangjiawei/DUDyConv into ``baseline/_ref/`` (git-ignored; it travels with
the working tree to GPU machines). ``tests/test_gpu_reference_dropin.py`` then imports
them with this library's compiled binding registered as ``cuda_ops_ext``, so the
reference's own Python code runs on these kernels. Only ``.py`` files are copied: the
reference's CUDA sources are neither needed nor built.
"""

from __future__ import annotations

import glob
import os
import shutil
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FILES = [
    "backbone_dil_unshared.py",
    "convtransformer_dil_unshared.py",
    "test_fused_dynamic_conv_against_reference.py",
    "test_fused_source_conv_mixed.py",
]


def stage(src: str, dst: str) -> list[str]:
    os.makedirs(os.path.join(dst, "cuda_ops"), exist_ok=True)
    done = []
    for f in FILES + [os.path.relpath(p, src) for p in glob.glob(os.path.join(src, "cuda_ops", "*.py"))]:
        shutil.copyfile(os.path.join(src, f), os.path.join(dst, f))
        done.append(f)
    return done


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit(__doc__)
    dst = sys.argv[2] if len(sys.argv) > 2 else os.path.join(ROOT, "baseline", "_ref")
    for f in stage(sys.argv[1], dst):
        print("staged", f)
