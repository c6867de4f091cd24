"""Loader and C-ABI signatures of the in-tree sm_100a kernel library (``lib/libdt_kernels.so``).

The library exports plain ``extern "C"`` launchers that take raw device pointers and a
``cudaStream_t``; every wrapper here passes ``tensor.data_ptr()`` and the current torch stream, so the
calls are recorded correctly inside ``torch.cuda.graph`` capture. A missing or failing library raises
immediately: there is no silent PyTorch fallback on the CUDA path.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from .. import _build

_LIB = None
_LOCK = threading.Lock()

c_int, c_ll, c_float, c_void = ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_void_p

# name -> argtypes (all return int status)
_SIGS = {
    "dt_get_error": [c_void, c_void, c_void],
    "dt_clear_error": [c_void],
    "dt_device_sm_count": [c_int],
    "dt_gemm_bf16": [c_void, c_int, c_ll, c_void, c_int, c_ll, c_void, c_ll, c_int, c_int, c_int, c_int, c_float,
                     c_int, c_int, c_void],
    "dt_gemm_bf16_peer": [c_void, c_int, c_ll, c_void, c_int, c_ll, c_void, c_ll, c_int, c_int, c_int, c_float, c_int,
                          c_void, c_void, c_void, c_void],
    "dt_add_rmsnorm_fwd_tp": [c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_int, c_int, c_float,
                              c_void, c_void, c_void, c_void],
    "dt_rmsnorm_bwd_tp": [c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_void,
                          c_int, c_int, c_void, c_void, c_void, c_void],
    "dt_add_rmsnorm_fwd": [c_void, c_void, c_void, c_void, c_int, c_int, c_void, c_void, c_void, c_void, c_void,
                           c_int, c_int, c_float, c_void],
    "dt_rmsnorm_bwd": [c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_int, c_int,
                       c_void],
    "dt_embedding_bwd": [c_void, c_void, c_int, c_int, c_void, c_int, c_int, c_void],
    "dt_rope_fwd": [c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_int, c_void],
    "dt_rope_bwd": [c_void, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_int, c_void],
    "dt_swiglu_fwd": [c_void, c_void, c_ll, c_int, c_void],
    "dt_gemm_qkv_rope": [c_void, c_ll, c_void, c_ll, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int,
                         c_int, c_int, c_int, c_void],
    "dt_gemm_swiglu_fwd": [c_void, c_ll, c_void, c_ll, c_void, c_void, c_int, c_int, c_int, c_void],
    "dt_gemm_swiglu_bwd": [c_void, c_ll, c_void, c_ll, c_void, c_void, c_int, c_int, c_int, c_int, c_void],
    "dt_swiglu_bwd": [c_void, c_void, c_void, c_ll, c_int, c_void],
    "dt_ce_fwd_bwd": [c_void, c_ll, c_void, c_int, c_int, c_ll, c_ll, c_void, c_int, c_float, c_void],
    "dt_loss_reduce": [c_void, c_ll, c_float, c_void, c_void, c_void],
    "dt_gemm_logits_lse": [c_void, c_ll, c_void, c_ll, c_void, c_ll, c_int, c_int, c_int, c_void, c_void, c_void,
                           c_int, c_int, c_ll, c_void],
    "dt_ce_lse_bwd": [c_void, c_ll, c_void, c_int, c_ll, c_void, c_void, c_int, c_int, c_ll, c_void, c_int, c_float,
                      c_void, c_void],
    "dt_adamw_step": [c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_int, c_void, c_int, c_void,
                      c_void, c_void],
    "dt_adamw_apply": [c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_int, c_void, c_int, c_void,
                       c_void, c_void],
    "dt_seg_sqnorm": [c_void, c_void, c_void, c_void, c_int, c_void, c_int, c_void],
    "dt_cast_bf16": [c_void, c_void, c_ll, c_void],
}


class KernelError(RuntimeError):
    pass


# Kernel launches issued through this library (incremented per launcher call by the number of
# kernels that launcher starts); a CUDA-graph replay adds the count recorded at capture.
LAUNCHES = [0]
_KERNELS_PER_CALL = {"dt_adamw_step": 3, "dt_adamw_apply": 2, "dt_seg_sqnorm": 1, "dt_get_error": 0, "dt_clear_error": 0,
                    "dt_dm_fused": 2}


def lib():
    """Load (building first if the sources are newer) the kernel library."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = _build.KERNELS_SO
        if _build.kernels_stale():
            if os.environ.get("DT_NO_BUILD"):
                raise KernelError(f"kernel library {path} is missing or stale and DT_NO_BUILD is set")
            _build.build_kernels()
        L = ctypes.CDLL(path)
        for name, args in _SIGS.items():
            f = getattr(L, name, None)
            if f is None:
                continue
            f.argtypes = args
            f.restype = c_int
        L.dt_cuda_error_string.restype = ctypes.c_char_p
        L.dt_cuda_error_string.argtypes = [c_int]
        _check_driver(L)
        _LIB = L
        return L


MIN_DRIVER = 12080  # sm_100a code needs a CUDA 12.8+ driver


def _check_driver(L):
    """Fail with a clear message when a GPU is present but its driver cannot run sm_100a code (the role the
    reference's node/cli/cuda_compat.c plays for its own toolchain)."""
    if not hasattr(L, "dt_cuda_versions"):
        return
    drv, rt = ctypes.c_int(0), ctypes.c_int(0)
    L.dt_cuda_versions.argtypes = [ctypes.POINTER(c_int), ctypes.POINTER(c_int)]
    L.dt_cuda_versions(ctypes.byref(drv), ctypes.byref(rt))
    if 0 < drv.value < MIN_DRIVER:
        raise KernelError(f"CUDA driver {drv.value // 1000}.{drv.value % 1000 // 10} is older than 12.8, the "
                          f"minimum for sm_100a (B200) code built with CUDA {rt.value // 1000}.{rt.value % 1000 // 10}")


def register(name: str, argtypes, restype=c_int):
    """Declare the signature of an additional exported symbol."""
    f = getattr(lib(), name)
    f.argtypes = argtypes
    f.restype = restype
    return f


def check(rc: int, what: str):
    LAUNCHES[0] += _KERNELS_PER_CALL.get(what, 1)
    if rc != 0:
        msg = lib().dt_cuda_error_string(rc).decode() if rc > 0 else f"argument error {rc}"
        raise KernelError(f"{what} failed: {msg}")


def stream_ptr(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def device_error(stream=None):
    """Return (code, site) of the first device-side failure recorded by any kernel (0 = none)."""
    code, site = ctypes.c_int(0), ctypes.c_int(0)
    check(lib().dt_get_error(ctypes.byref(code), ctypes.byref(site), stream_ptr(stream)), "dt_get_error")
    return code.value, site.value


def clear_device_error(stream=None):
    check(lib().dt_clear_error(stream_ptr(stream)), "dt_clear_error")
