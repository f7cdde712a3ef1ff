"""Build the in-tree native libraries of dudyconv_b200.

* ``libdudyconv_b200.so``  -- the CUDA kernels and the C ABI (include/dudyconv_b200.h),
  compiled by nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``).
* ``cuda_ops_ext.*.so``    -- the thin torch binding: the reference's pybind module
  ``cuda_ops_ext`` (10 functions) and ``TORCH_LIBRARY(fused_source_conv_mixed)``
  (14 ops), calling the C ABI. Built with g++ against torch's headers.

Both land next to this file (git-ignored build outputs that travel with the tree).
Run ``python -m dudyconv_b200.build`` or call ``build()``. Rebuilds only what changed.
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import hashlib
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libdudyconv_b200.so")
EXT_NAME = "cuda_ops_ext"


def _cuda_home() -> str:
    return os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _nvcc() -> str:
    return os.path.join(_cuda_home(), "bin", "nvcc")


NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]


def _digest(paths, extra: str) -> str:
    h = hashlib.sha256(extra.encode())
    for p in sorted(paths):
        with open(p, "rb") as f:
            h.update(p.encode())
            h.update(f.read())
    return h.hexdigest()


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def _run(cmd, cwd=None):
    r = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build_lib(verbose: bool = False, jobs: int | None = None) -> str:
    """Compile csrc/*.cu with nvcc into libdudyconv_b200.so (incremental)."""
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr = _headers()
    objs = []
    todo = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        stamp = obj + ".sha"
        dig = _digest([src] + hdr, " ".join(NVCC_FLAGS))
        objs.append(obj)
        if os.path.exists(obj) and os.path.exists(stamp) and open(stamp).read() == dig:
            continue
        todo.append((src, obj, stamp, dig))

    def compile_one(item):
        src, obj, stamp, dig = item
        cmd = [_nvcc(), *NVCC_FLAGS, "-Xptxas", "-v", "-c", src, "-o", obj]
        out = _run(cmd)
        with open(stamp, "w") as f:
            f.write(dig)
        with open(obj + ".ptxas.txt", "w") as f:
            f.write(out)
        return src, out

    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
            for src, out in ex.map(compile_one, todo):
                if verbose:
                    print(f"[nvcc] {os.path.basename(src)}")
    link_dig = _digest(objs, "link")
    link_stamp = os.path.join(BUILD, "lib.sha")
    if todo or not os.path.exists(LIB) or not os.path.exists(link_stamp) or \
            open(link_stamp).read() != link_dig:
        _run([_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs,
              "-o", LIB, "-lcudart_static", "-lrt", "-ldl", "-lpthread"])
        with open(link_stamp, "w") as f:
            f.write(link_dig)
        if verbose:
            print(f"[link] {LIB}")
    return LIB


def _ext_path() -> str:
    return os.path.join(PKG, EXT_NAME + sysconfig.get_config_var("EXT_SUFFIX"))


def build_ext(verbose: bool = False) -> str:
    """Compile csrc/torch_ext.cpp into the cuda_ops_ext Python module."""
    import torch
    from torch.utils import cpp_extension

    src = os.path.join(CSRC, "torch_ext.cpp")
    out = _ext_path()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    flags = [
        "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={EXT_NAME}",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
    ]
    incs = [f"-I{p}" for p in cpp_extension.include_paths(device_type="cuda")]
    incs += [f"-I{sysconfig.get_paths()['include']}", f"-I{os.path.join(_cuda_home(), 'include')}",
             f"-I{os.path.join(ROOT, 'include')}"]
    libdirs = [f"-L{p}" for p in cpp_extension.library_paths(device_type="cuda")]
    libs = ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
            f"-L{PKG}", "-ldudyconv_b200", "-Wl,-rpath,$ORIGIN"]
    dig = _digest([src, LIB] + _headers(), " ".join(flags) + torch.__version__)
    stamp = os.path.join(BUILD, "ext.sha")
    if os.path.exists(out) and os.path.exists(stamp) and open(stamp).read() == dig:
        return out
    os.makedirs(BUILD, exist_ok=True)
    _run(["g++", *flags, *incs, src, "-o", out, *libdirs, *libs])
    with open(stamp, "w") as f:
        f.write(dig)
    if verbose:
        print(f"[g++] {out}")
    return out


def build(verbose: bool = False) -> None:
    build_lib(verbose=verbose)
    build_ext(verbose=verbose)


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
