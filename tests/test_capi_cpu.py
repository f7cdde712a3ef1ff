"""C ABI checks that need no GPU: the library loads, exports every entry point that
include/dudyconv_b200.h declares, and its host-side logic (plan legality and the
reference heuristics, argument validation, workspace sizing) behaves as specified."""

import ctypes
import os
import re

import pytest

from dudyconv_b200 import capi


def _header_symbols():
    text = open(capi.HEADER_PATH).read()
    return sorted(set(re.findall(r"^DUDY_API[^;(]*?\b(dudy_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    syms = _header_symbols()
    assert len(syms) >= 16
    lib = capi.lib()
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in the header but not exported"
    # the ctypes signature table covers the whole header
    assert sorted(capi.SIGNATURES) == syms


def test_version_and_plan_names():
    lib = capi.lib()
    assert b"sm_100a" in lib.dudy_version()
    assert lib.dudy_fdc_plan_name(-1) == b"not_cached"
    assert lib.dudy_fdc_plan_name(capi.PLAN_SIMT) == b"simt_generic"
    assert lib.dudy_fdc_plan_name(capi.PLAN_TC) == b"tcgen05_tmem"


@pytest.mark.parametrize("plan,D,C,S,off,dil,want", [
    (0, 17, 5, 4, 0, 2, 1),
    (1, 16, 8, 3, 0, 1, 1), (1, 16, 8, 4, 0, 1, 0),
    (2, 64, 32, 3, 0, 1, 1), (2, 64, 16, 3, 0, 1, 0),
    (3, 256, 16, 3, 0, 1, 1), (3, 128, 16, 3, 0, 1, 0),
    (100, 16, 8, 3, 2, 1, 1), (100, 16, 8, 3, 1, 1, 0),
    (101, 16, 8, 3, 8, 4, 1), (101, 16, 8, 3, 7, 4, 0),
    (103, 256, 16, 3, 64, 1, 1), (103, 256, 16, 3, 64, 64, 0),
    (7, 256, 16, 3, 0, 1, 0),
])
def test_fscm_forward_plan_legality(plan, D, C, S, off, dil, want):
    # rules of fused_source_conv_mixed_forward.cu:309-365
    assert capi.lib().dudy_fscm_forward_plan_legal(plan, D, C, S, off, dil) == want


def test_fscm_heuristics():
    lib = capi.lib()
    assert lib.dudy_fscm_forward_default_plan(1, 256, 512, 16, 3, 0, 256, 1) == 3
    assert lib.dudy_fscm_forward_default_plan(1, 256, 512, 16, 3, 64, 256, 1) == 103
    assert lib.dudy_fscm_forward_default_plan(1, 64, 512, 8, 3, 0, 256, 1) == 1
    assert lib.dudy_fscm_forward_default_plan(1, 64, 512, 7, 5, 0, 256, 1) == 0
    # backward: atomic for C > 64, tiny problems; gather-x when the affected range covers L
    assert lib.dudy_fscm_backward_default_plan(1, 64, 512, 65, 3, 0, 256, 1) == 0
    assert lib.dudy_fscm_backward_default_plan(1, 4, 64, 8, 3, 0, 32, 1) == 0
    assert lib.dudy_fscm_backward_default_plan(1, 256, 512, 16, 3, 0, 512, 1) == 2
    assert lib.dudy_fscm_backward_default_plan(1, 256, 8192, 16, 3, 0, 1024, 1) == 1
    assert lib.dudy_fscm_backward_plan_legal(1, 64, 8, 128) == 1
    assert lib.dudy_fscm_backward_plan_legal(2, 65, 8, 128) == 0
    assert lib.dudy_fscm_backward_plan_legal(1, 16, 3, 0) == 0
    assert lib.dudy_fscm_backward_plan_legal(0, 1000, 100, 0) == 1


def test_fdc_validation_messages_without_gpu():
    lib = capi.lib()
    fake = ctypes.c_void_p(256)
    # t_offset + T > L: rejected before any device work (reference message)
    rc = lib.dudy_fdc_forward(fake, fake, fake, fake, 1, 16, 64, 32, 4, 3, 40, 1, 1, -1, None)
    assert rc == capi.ERR_INVALID
    assert "t_offset + T must be <= L" in capi.last_error()
    rc = lib.dudy_fdc_forward(fake, fake, fake, fake, 1, 16, 64, 32, 4, 3, 0, 0, 1, -1, None)
    assert rc == capi.ERR_INVALID and "dilation must be positive." == capi.last_error()
    rc = lib.dudy_fdc_forward(fake, fake, fake, fake, 1, 16, 64, 32, 4, 3, -1, 1, 1, -1, None)
    assert rc == capi.ERR_INVALID and "t_offset must be non-negative." == capi.last_error()
    rc = lib.dudy_fdc_forward(fake, fake, fake, fake, 1, 16, 64, 32, 4, 3, 0, 1, 7, -1, None)
    assert rc == capi.ERR_INVALID
    # valid arguments on a machine without an sm_100 device: a device error, not a crash
    import torch
    if not torch.cuda.is_available():
        rc = lib.dudy_fdc_forward(fake, fake, fake, fake, 1, 16, 64, 32, 4, 3, 0, 1, 1, -1, None)
        assert rc == capi.ERR_DEVICE


def test_workspace_sizes():
    lib = capi.lib()
    ws = lib.dudy_fdc_backward_workspace_size(16, 256, 4096, 4096, 128, 3, 0, 1, 1, -1)
    assert ws > 0 and ws % 256 == 0
    # tensor-core partials of grad_mix: one fp32 [D,N] slice per CTA (at most 148 on B200)
    assert ws >= 256 * 128 * 4
    assert lib.dudy_fdc_backward_workspace_size(1, 16, 64, 80, 4, 3, 0, 1, 1, -1) == 0  # invalid
    ws2 = lib.dudy_fscm_backward_workspace_size(2, 64, 256, 8, 3, 64, 128, 1, 1, 1, 64)
    assert ws2 > 0 and ws2 % 256 == 0


def test_peer_exchange_struct_layout_matches_header(tmp_path):
    """The ctypes mirror of DudyPeerExchange has the C compiler's size and offsets."""
    import ctypes
    import shutil
    import subprocess

    from dudyconv_b200 import capi

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "dudyconv_b200.h"\n'
        "int main(void) { printf(\"%zu %zu %zu %zu %d\\n\", sizeof(DudyPeerExchange),"
        " offsetof(DudyPeerExchange, rank), offsetof(DudyPeerExchange, world),"
        " offsetof(DudyPeerExchange, epoch), DUDY_MAX_PEERS); return 0; }\n")
    exe = tmp_path / "layout"
    inc = os.path.join(os.path.dirname(capi.HEADER_PATH))
    subprocess.run([cc, "-I", inc, str(src), "-o", str(exe)], check=True)
    got = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    want = [ctypes.sizeof(capi.PeerExchange), capi.PeerExchange.rank.offset,
            capi.PeerExchange.world.offset, capi.PeerExchange.epoch.offset, capi.MAX_PEERS]
    assert [int(v) for v in got] == want
