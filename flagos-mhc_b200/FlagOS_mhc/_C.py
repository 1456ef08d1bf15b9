"""ctypes binding of libmhc_b200.so (the C ABI declared in include/mhc_b200.h).

The library is loaded once, on first use.  There is no fallback: if the shared
library is missing or the tensors are not on an sm_100 GPU, the call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libmhc_b200.so")
_lib = None
_lock = threading.Lock()

MHC_F32, MHC_F16, MHC_BF16 = 0, 1, 2
_DTYPE = {torch.float32: MHC_F32, torch.float16: MHC_F16, torch.bfloat16: MHC_BF16}

MHC_OK = 0
MHC_ERR_INVALID_ARGUMENT = 1
MHC_ERR_UNSUPPORTED_N = 2
MHC_ERR_UNSUPPORTED_DTYPE = 3
MHC_ERR_WORKSPACE = 4
MHC_ERR_CUDA = 5
MHC_ERR_DEVICE = 6
MHC_ERR_TIMEOUT = 7
MHC_ERR_SCRATCH_LIMIT = 8

_vp, _fp = ctypes.c_void_p, ctypes.c_void_p
_i64, _i32, _f32, _sz = ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_size_t

_SIGS = {
    "mhc_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "mhc_version": (ctypes.c_int, []),
    "mhc_kernel_launches": (ctypes.c_uint64, []),
    "mhc_device_status": (ctypes.c_int, []),
    "mhc_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_uint32, _vp]),
    "mhc_post_fwd": (ctypes.c_int, [_vp, _fp, _vp, _fp, _vp, _i64, _i32, _i64, _i32, _vp]),
    "mhc_post_bwd": (ctypes.c_int, [_vp, _vp, _fp, _vp, _fp, _vp, _fp, _vp, _fp, _i64, _i32,
                                    _i64, _i32, _vp]),
    "mhc_pre_fwd_workspace_bytes": (_sz, [_i64, _i32, _i64, _i32]),
    "mhc_pre_fwd": (ctypes.c_int, [_vp, _fp, _fp, _fp, _i64, _i32, _i64, _i32, _f32, _f32, _f32,
                                   _f32, _i32, _vp, _fp, _fp, _fp, _fp, _fp, _fp, _fp, _vp, _sz,
                                   _vp]),
    "mhc_pre_fwd_noalloc": (ctypes.c_int, [_vp, _fp, _fp, _fp, _i64, _i32, _i64, _i32, _f32, _f32,
                                           _f32, _f32, _i32, _vp, _fp, _fp, _fp, _fp, _fp, _fp,
                                           _fp, _vp]),
    "mhc_pre_bwd_workspace_bytes": (_sz, [_i64, _i32, _i64, _i32, _i32]),
    "mhc_pre_bwd": (ctypes.c_int, [_vp, _fp, _fp, _fp, _fp, _fp, _fp, _vp, _fp, _fp, _i64, _i32,
                                   _i64, _i32, _f32, _f32, _f32, _f32, _i32, _vp, _fp, _fp, _fp,
                                   _vp, _sz, _vp]),
    "mhc_post_fwd_strided": (ctypes.c_int, [_vp, _i64, _fp, _vp, _i64, _fp, _vp, _i64, _i32, _i64,
                                            _i32, _vp]),
    "mhc_post_bwd_strided": (ctypes.c_int, [_vp, _i64, _vp, _i64, _fp, _vp, _i64, _fp, _vp, _fp,
                                            _vp, _fp, _i64, _i32, _i64, _i32, _vp]),
    "mhc_pre_fwd_strided": (ctypes.c_int, [_vp, _i64, _fp, _fp, _fp, _i64, _i32, _i64, _i32, _f32,
                                           _f32, _f32, _f32, _i32, _vp, _fp, _fp, _fp, _fp, _fp,
                                           _fp, _fp, _vp, _sz, _vp]),
    "mhc_pre_bwd_strided": (ctypes.c_int, [_vp, _i64, _fp, _fp, _fp, _fp, _fp, _fp, _vp, _i64, _fp,
                                           _fp, _i64, _i32, _i64, _i32, _f32, _f32, _f32, _f32,
                                           _i32, _vp, _vp, _fp, _fp, _fp, _vp, _sz, _vp]),
    "mhc_post_fwd_mix_supported": (ctypes.c_int, [_i64, _i32, _i64, _i32]),
    "mhc_post_fwd_mix_layers": (_i32, [_i64, _i32, _i64, _i32]),
    "mhc_post_fwd_mix_workspace_bytes": (_sz, [_i64, _i32, _i64, _i32]),
    "mhc_post_fwd_mix": (ctypes.c_int, [_vp, _fp, _vp, _fp, _vp, _i64, _i32, _i64, _i32, _fp, _fp,
                                        _vp, _sz, _vp]),
    "mhc_pre_fwd_premixed": (ctypes.c_int, [_vp, _fp, _i32, _fp, _fp, _i64, _i32, _i64, _i32,
                                            _f32, _f32, _f32, _f32, _i32, _vp, _fp, _fp, _fp,
                                            _fp, _fp, _fp, _fp, _vp]),
    "mhc_peer_region_bytes": (_sz, [_i64]),
    "mhc_peer_region_alloc": (ctypes.c_int, [_i64, ctypes.POINTER(ctypes.c_void_p)]),
    "mhc_peer_region_free": (ctypes.c_int, [_vp]),
    "mhc_peer_handle_bytes": (ctypes.c_int, []),
    "mhc_peer_handle": (ctypes.c_int, [_vp, ctypes.c_char_p]),
    "mhc_peer_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "mhc_peer_close": (ctypes.c_int, [_vp]),
    "mhc_grad_sum_peers": (ctypes.c_int, [_vp, _vp, _i64, ctypes.POINTER(ctypes.c_void_p), _i32,
                                          _i32, ctypes.c_uint32, ctypes.c_uint64, _vp]),
    "mhc_pre_bwd_accumulate": (ctypes.c_int, [_vp, _fp, _fp, _fp, _fp, _fp, _fp, _vp, _fp, _fp,
                                              _i64, _i32, _i64, _i32, _f32, _f32, _f32, _f32,
                                              _i32, _vp, _vp, _fp, _fp, _fp, _vp, _sz, _vp]),
}


def lib_path() -> str:
    return _LIB_PATH


def lib():
    """Load (once) and return the ctypes handle; raise if the library is absent."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(_LIB_PATH):
                    raise RuntimeError(
                        f"FlagOS_mhc: CUDA library not found at {_LIB_PATH}; build it with "
                        "`python flagos-mhc_b200/build.py` (there is no CPU fallback)")
                h = ctypes.CDLL(_LIB_PATH)
                for name, (res, args) in _SIGS.items():
                    fn = getattr(h, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = h
    return _lib


def token_view(t, inner_dims, inner_numel):
    """Token stride (in elements) of t viewed as (tokens, *inner) without a copy, or None.

    t is (T, *inner) or (B, S, *inner) with the `inner_dims` trailing dims packed
    (their numel is `inner_numel`); for 4D/3D-with-B,S the B stride must equal S times
    the S stride so that the B*S tokens share one stride."""
    lead = t.dim() - inner_dims
    if lead not in (1, 2) or t.numel() == 0:
        return None
    inner = t.shape[lead:]
    expect = 1
    for d in range(t.dim() - 1, lead - 1, -1):
        if inner[d - lead] != 1 and t.stride(d) != expect:
            return None
        expect *= t.shape[d]
    if lead == 1:
        ts = t.stride(0)
    else:
        B, S = t.shape[0], t.shape[1]
        ts = t.stride(1) if S > 1 else t.stride(0)
        if B > 1 and S > 1 and t.stride(0) != S * t.stride(1):
            return None
    if t.shape[0] * (t.shape[1] if lead == 2 else 1) > 1 and ts < inner_numel:
        return None
    return max(int(ts), inner_numel)


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def dtype_code(dt):
    try:
        return _DTYPE[dt]
    except KeyError:
        raise TypeError(f"FlagOS_mhc: unsupported dtype {dt}; expected float32/float16/bfloat16")


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def check(status: int, what: str):
    if status == MHC_OK:
        return
    msg = lib().mhc_status_string(status).decode()
    text = f"FlagOS_mhc.{what}: {msg} (status {status})"
    if status == MHC_ERR_UNSUPPORTED_N:
        raise NotImplementedError(text)
    if status in (MHC_ERR_INVALID_ARGUMENT, MHC_ERR_UNSUPPORTED_DTYPE):
        raise ValueError(text)
    raise RuntimeError(text)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("FlagOS_mhc: operators run only on CUDA (sm_100) tensors; "
                               f"got a tensor on {t.device}")
