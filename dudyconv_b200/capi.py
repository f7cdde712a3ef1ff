"""ctypes binding of the C ABI in ``include/dudyconv_b200.h`` (libdudyconv_b200.so).

This is the reference-facing boundary with plain pointers and sizes; the parity tests
call it directly, and it is the binding a non-torch host (or a ctypes-based caller)
would use. Tensor arguments may be torch tensors (their ``data_ptr()`` is passed) or
raw integer device addresses.
"""

from __future__ import annotations

import ctypes
import os

from . import PKG_DIR

LIB_PATH = os.path.join(PKG_DIR, "libdudyconv_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(PKG_DIR), "include", "dudyconv_b200.h")

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE, ERR_DEVICE = 0, 1, 2, 3, 4, 5
PLAN_AUTO, PLAN_SIMT, PLAN_TC = -1, 100, 200

_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_int = ctypes.c_int
_sz = ctypes.c_size_t

MAX_PEERS = 8


class PeerExchange(ctypes.Structure):
    """DudyPeerExchange of the C ABI (the data-parallel backward's peer buffers)."""
    _fields_ = [("bufs", ctypes.c_void_p * MAX_PEERS), ("rank", ctypes.c_int),
                ("world", ctypes.c_int), ("epoch", ctypes.c_uint32)]


# name -> (restype, argtypes)
SIGNATURES = {
    "dudy_version": (ctypes.c_char_p, []),
    "dudy_last_error": (ctypes.c_char_p, []),
    "dudy_device_error": (_int, [_int]),
    "dudy_device_error_info": (_int, [ctypes.POINTER(ctypes.c_int), _int]),
    "dudy_fdc_plan_name": (ctypes.c_char_p, [_int]),
    "dudy_fdc_default_plan": (_int, [_vp, _vp, _vp] + [_i64] * 8 + [_int]),
    "dudy_fdc_plan_available": (_int, [_int, _vp, _vp, _vp] + [_i64] * 8 + [_int]),
    "dudy_fdc_forward": (_int, [_vp] * 4 + [_i64] * 8 + [_int, _int, _vp]),
    "dudy_fdc_backward_workspace_size": (_sz, [_i64] * 8 + [_int, _int]),
    "dudy_fdc_backward": (_int, [_vp] * 8 + [_sz] + [_i64] * 8 + [_int, _int, _vp]),
    "dudy_fdc_backward_grad_h": (_int, [_vp] * 4 + [_i64] * 8 + [_int, _int, _vp]),
    "dudy_fdc_backward_grad_kc_mix": (_int, [_vp] * 7 + [_sz] + [_i64] * 8 + [_int, _int, _vp]),
    "dudy_fdc_backward_noalloc": (_int, [_vp] * 7 + [_i64] * 8 + [_int, _int, _vp]),
    "dudy_fscm_forward_plan_legal": (_int, [_int] + [_i64] * 5),
    "dudy_fscm_forward_default_plan": (_int, [_i64] * 8),
    "dudy_fscm_forward": (_int, [_vp] * 6 + [_i64] * 8 + [_int, _int, _vp]),
    "dudy_fscm_backward_plan_legal": (_int, [_int, _i64, _i64, _i64]),
    "dudy_fscm_backward_default_plan": (_int, [_i64] * 8),
    "dudy_fscm_backward_workspace_size": (_sz, [_i64] * 8 + [_int, _int, _i64]),
    "dudy_fscm_backward": (_int, [_vp] * 12 + [_sz] + [_i64] * 8 + [_int, _int, _i64, _vp]),
    "dudy_check_phi_approx": (_int, [_vp]),
    "dudy_selftest_wait_timeout": (_int, [_int, ctypes.POINTER(ctypes.c_int)]),
    "dudy_logits_to_kernel": (_int, [_vp, _vp] + [_i64] * 4 + [_int, _vp]),
    "dudy_fdc_exchange_bytes": (_sz, [_i64, _i64]),
    "dudy_fdc_backward_dp": (_int, [_vp] * 8 + [_sz, ctypes.POINTER(PeerExchange)] + [_i64] * 8
                             + [_int, _int, _vp]),
    "dudy_fdc_backward_dp_deferred": (_int, [_vp] * 9 + [_sz, ctypes.POINTER(PeerExchange)]
                                      + [_i64] * 8 + [_int, _int, _vp]),
    "dudy_fdc_exchange_finish": (_int, [ctypes.POINTER(PeerExchange), _vp, _i64, _i64, _int, _vp]),
    "dudy_logits_to_kernel_backward": (_int, [_vp] * 3 + [_i64] * 4 + [_int, _vp]),
}

_LIB = None


class DudyError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{msg} (status {status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libdudyconv_b200.so and declare every exported entry point."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run `python -m dudyconv_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


_DTYPE_CODES = None


def dtype_code(t) -> int:
    global _DTYPE_CODES
    if _DTYPE_CODES is None:
        import torch
        _DTYPE_CODES = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16,
                        torch.bfloat16: DTYPE_BF16}
    return _DTYPE_CODES[t.dtype]


def last_error() -> str:
    return lib().dudy_last_error().decode()


def _check(rc: int):
    if rc != OK:
        raise DudyError(rc, last_error())


def fdc_forward(h, kc, mix, out, off: int, dilation: int, plan: int = PLAN_AUTO, stream=None):
    B, D, L = h.shape
    _, K, N, T = kc.shape
    _check(lib().dudy_fdc_forward(_ptr(h), _ptr(kc), _ptr(mix), _ptr(out), B, D, L, T, N, K,
                                  off, dilation, dtype_code(h), plan, _stream(stream)))


def fdc_backward_workspace_size(h, kc, off: int, dilation: int, plan: int = PLAN_AUTO) -> int:
    B, D, L = h.shape
    _, K, N, T = kc.shape
    return int(lib().dudy_fdc_backward_workspace_size(B, D, L, T, N, K, off, dilation,
                                                      dtype_code(h), plan))


def fdc_backward(go, h, kc, mix, grad_h, grad_kc, grad_mix, workspace, off: int, dilation: int,
                 plan: int = PLAN_AUTO, stream=None):
    B, D, L = h.shape
    _, K, N, T = kc.shape
    ws_bytes = workspace.numel() * workspace.element_size()
    _check(lib().dudy_fdc_backward(_ptr(go), _ptr(h), _ptr(kc), _ptr(mix), _ptr(grad_h),
                                   _ptr(grad_kc), _ptr(grad_mix), _ptr(workspace), ws_bytes,
                                   B, D, L, T, N, K, off, dilation, dtype_code(h), plan,
                                   _stream(stream)))


def fdc_backward_grad_h(go, kc, mix, grad_h, off: int, dilation: int, plan: int = PLAN_AUTO,
                        stream=None):
    B, D, L = grad_h.shape
    _, K, N, T = kc.shape
    _check(lib().dudy_fdc_backward_grad_h(_ptr(go), _ptr(kc), _ptr(mix), _ptr(grad_h), B, D, L,
                                          T, N, K, off, dilation, dtype_code(go), plan,
                                          _stream(stream)))


def fdc_backward_grad_kc_mix(go, h, kc, mix, grad_kc, grad_mix, workspace, off: int,
                             dilation: int, plan: int = PLAN_AUTO, stream=None):
    B, D, L = h.shape
    _, K, N, T = kc.shape
    ws_bytes = workspace.numel() * workspace.element_size()
    _check(lib().dudy_fdc_backward_grad_kc_mix(_ptr(go), _ptr(h), _ptr(kc), _ptr(mix),
                                               _ptr(grad_kc), _ptr(grad_mix), _ptr(workspace),
                                               ws_bytes, B, D, L, T, N, K, off, dilation,
                                               dtype_code(h), plan, _stream(stream)))


def fdc_backward_noalloc(go, h, kc, mix, grad_h, grad_kc, grad_mix, off: int, dilation: int,
                         plan: int = PLAN_AUTO, stream=None):
    """Backward with the library's fixed scratch array instead of a caller workspace."""
    B, D, L = h.shape
    _, K, N, T = kc.shape
    _check(lib().dudy_fdc_backward_noalloc(_ptr(go), _ptr(h), _ptr(kc), _ptr(mix), _ptr(grad_h),
                                           _ptr(grad_kc), _ptr(grad_mix), B, D, L, T, N, K, off,
                                           dilation, dtype_code(h), plan, _stream(stream)))


def fdc_default_plan(h, kc, mix, off: int, dilation: int) -> int:
    B, D, L = h.shape
    _, K, N, T = kc.shape
    return int(lib().dudy_fdc_default_plan(_ptr(h), _ptr(kc), _ptr(mix), B, D, L, T, N, K, off,
                                           dilation, dtype_code(h)))


def fscm_forward(x, weight, bias, mix_w, mix_b, out, off: int, T: int, dilation: int,
                 plan: int = PLAN_AUTO, stream=None):
    B, D, L = x.shape
    _, C, S = weight.shape
    _check(lib().dudy_fscm_forward(_ptr(x), _ptr(weight), _ptr(bias), _ptr(mix_w), _ptr(mix_b),
                                   _ptr(out), B, D, L, C, S, off, T, dilation, dtype_code(x),
                                   plan, _stream(stream)))


def fscm_backward_workspace_size(x, weight, off: int, T: int, dilation: int,
                                 plan: int = PLAN_AUTO, tile_t: int = 0) -> int:
    B, D, L = x.shape
    _, C, S = weight.shape
    return int(lib().dudy_fscm_backward_workspace_size(B, D, L, C, S, off, T, dilation,
                                                       dtype_code(x), plan, tile_t))


def fscm_backward(go, x, weight, bias, mix_w, mix_b, grad_x, grad_w, grad_bias, grad_mix_w,
                  grad_mix_b, workspace, off: int, T: int, dilation: int, plan: int = PLAN_AUTO,
                  tile_t: int = 0, stream=None):
    B, D, L = x.shape
    _, C, S = weight.shape
    ws_bytes = workspace.numel() * workspace.element_size()
    _check(lib().dudy_fscm_backward(_ptr(go), _ptr(x), _ptr(weight), _ptr(bias), _ptr(mix_w),
                                    _ptr(mix_b), _ptr(grad_x), _ptr(grad_w), _ptr(grad_bias),
                                    _ptr(grad_mix_w), _ptr(grad_mix_b), _ptr(workspace),
                                    ws_bytes, B, D, L, C, S, off, T, dilation, dtype_code(x),
                                    plan, tile_t, _stream(stream)))


def device_error(reset: bool = False) -> int:
    return int(lib().dudy_device_error(1 if reset else 0))


def device_error_info(reset: bool = False):
    """(site, block, thread, counter) of the first timed-out device wait; site 0 = none."""
    buf = (ctypes.c_int * 4)()
    lib().dudy_device_error_info(buf, 1 if reset else 0)
    return tuple(int(v) for v in buf)


def selftest_wait_timeout(limit_us: int = 2000):
    """Run the bounded-wait self-test kernel; returns (warp0 completed, warp1 completed)."""
    buf = (ctypes.c_int * 2)()
    _check(lib().dudy_selftest_wait_timeout(int(limit_us), buf))
    return int(buf[0]), int(buf[1])


def logits_to_kernel(logits, kc, stream=None):
    """kc [B,K,N,T] <- softmax over K of logits [B,N*K,T], flipped (kk = 0 current token)."""
    B, K, N, T = kc.shape
    _check(lib().dudy_logits_to_kernel(_ptr(logits), _ptr(kc), B, N, K, T, dtype_code(kc),
                                       _stream(stream)))


def logits_to_kernel_backward(kc, grad_kc, grad_logits, stream=None):
    B, K, N, T = kc.shape
    _check(lib().dudy_logits_to_kernel_backward(_ptr(kc), _ptr(grad_kc), _ptr(grad_logits), B, N,
                                                K, T, dtype_code(kc), _stream(stream)))


def fdc_exchange_bytes(D: int, N: int) -> int:
    return int(lib().dudy_fdc_exchange_bytes(D, N))


def fdc_backward_dp(go, h, kc, mix, grad_h, grad_kc, grad_mix, workspace, xchg: PeerExchange,
                    off: int, dilation: int, plan: int = PLAN_AUTO, stream=None):
    """dudy_fdc_backward_dp: the backward with grad_mix summed over the ranks of `xchg`."""
    B, D, L = h.shape
    _, K, N, T = kc.shape
    ws_bytes = workspace.numel() * workspace.element_size()
    _check(lib().dudy_fdc_backward_dp(_ptr(go), _ptr(h), _ptr(kc), _ptr(mix), _ptr(grad_h),
                                      _ptr(grad_kc), _ptr(grad_mix), _ptr(workspace), ws_bytes,
                                      ctypes.byref(xchg), B, D, L, T, N, K, off, dilation,
                                      dtype_code(h), plan, _stream(stream)))


def fdc_backward_dp_deferred(go, h, kc, mix, grad_h, grad_kc, grad_mix, grad_mix_prev, workspace,
                             xchg: PeerExchange, off: int, dilation: int, plan: int = PLAN_AUTO,
                             stream=None):
    """dudy_fdc_backward_dp_deferred: this rank's backward; grad_mix gets this rank's own sum,
    grad_mix_prev the sum over ranks of the previous call."""
    B, D, L = h.shape
    _, K, N, T = kc.shape
    ws_bytes = workspace.numel() * workspace.element_size()
    _check(lib().dudy_fdc_backward_dp_deferred(
        _ptr(go), _ptr(h), _ptr(kc), _ptr(mix), _ptr(grad_h), _ptr(grad_kc), _ptr(grad_mix),
        _ptr(grad_mix_prev), _ptr(workspace), ws_bytes, ctypes.byref(xchg), B, D, L, T, N, K,
        off, dilation, dtype_code(h), plan, _stream(stream)))


def fdc_exchange_finish(xchg: PeerExchange, grad_mix, stream=None):
    """dudy_fdc_exchange_finish: the sum over ranks of call xchg.epoch into grad_mix."""
    D, N = grad_mix.shape
    _check(lib().dudy_fdc_exchange_finish(ctypes.byref(xchg), _ptr(grad_mix), D, N,
                                          dtype_code(grad_mix), _stream(stream)))
