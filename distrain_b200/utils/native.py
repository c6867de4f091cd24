"""ctypes binding of the C++ runtime library (``lib/libdt_runtime.so``): codecs, shard assignment,
data loading and the coordinator's HTTP server core. CPU-only; builds on first use if stale."""
from __future__ import annotations

import ctypes
import os
import threading

from .. import _build

_RT = None
_LOCK = threading.Lock()
c_int, c_ll, c_ull, c_void, c_char_p, c_float = (ctypes.c_int, ctypes.c_longlong, ctypes.c_ulonglong, ctypes.c_void_p,
                                                  ctypes.c_char_p, ctypes.c_float)

_SIGS = {
    "dtr_last_error": ([], c_char_p),
    "dtr_blob_size": ([c_void], c_ll),
    "dtr_blob_data": ([c_void], c_void),
    "dtr_blob_free": ([c_void], None),
    "dtr_zstd_available": ([], c_int),
    "dtr_zstd_compress": ([c_void, c_ll, c_int], c_void),
    "dtr_zstd_decompress": ([c_void, c_ll], c_void),
    "dtr_siphash13": ([c_void, c_ll], c_ull),
    "dtr_splitmix64": ([c_ull], c_ull),
    "dtr_lowrank_omega": ([c_ll, c_ll, c_ll, c_void], None),
    "dtr_hash_str": ([c_char_p], c_ull),
    "dtr_hash_u64": ([c_ull], c_ull),
    "dtr_shard_assignment": ([c_char_p, c_ull, c_ll, c_ll, c_void], c_ll),
    "dtr_st_open": ([c_char_p], c_void),
    "dtr_st_open_bytes": ([c_void, c_ll], c_void),
    "dtr_st_close": ([c_void], None),
    "dtr_st_count": ([c_void], c_int),
    "dtr_st_name": ([c_void, c_int], c_char_p),
    "dtr_st_dtype": ([c_void, c_int], c_char_p),
    "dtr_st_ndim": ([c_void, c_int], c_int),
    "dtr_st_dim": ([c_void, c_int, c_int], c_ll),
    "dtr_st_metadata": ([c_void], c_char_p),
    "dtr_st_read_f32": ([c_void, c_int, c_void, c_ll], c_ll),
    "dtr_st_save": ([c_char_p, c_int, c_void, c_void, c_void, c_void, c_char_p, c_void], c_int),
    "dtr_sparse_delta_encode": ([c_int, c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_char_p, c_int],
                                c_void),
    "dtr_delta_decode": ([c_void, c_ll], c_void),
    "dtr_delta_free": ([c_void], None),
    "dtr_delta_is_lowrank": ([c_void], c_int),
    "dtr_delta_raw_json": ([c_void], c_char_p),
    "dtr_delta_count": ([c_void], c_int),
    "dtr_delta_name": ([c_void, c_int], c_char_p),
    "dtr_delta_ndim": ([c_void, c_int], c_int),
    "dtr_delta_dim": ([c_void, c_int, c_int], c_ll),
    "dtr_delta_data": ([c_void, c_int], c_void),
    "dtr_delta_numel": ([c_void, c_int], c_ll),
    "dtr_delta_config": ([c_void], c_char_p),
    "dtr_dtz_encode": ([c_ll, c_ll, c_void, c_void, c_void, c_void, c_int, c_int], c_void),
    "dtr_dtz_decode_dense": ([c_void, c_ll], c_void),
    "dts_accept_push": ([c_ll, c_ll, c_int, c_int, c_void, c_void, c_char_p, c_ll, ctypes.c_double, ctypes.c_double,
                         c_void, c_void, c_int], c_int),
    "dts_should_checkpoint": ([c_int, c_void, c_int, c_void, c_void, ctypes.c_double, c_int], c_int),
    "dts_update_round_time": ([ctypes.c_double, c_ll, c_ll], ctypes.c_double),
}


class NativeError(RuntimeError):
    pass


def rt():
    global _RT
    if _RT is not None:
        return _RT
    with _LOCK:
        if _RT is not None:
            return _RT
        if _build.runtime_stale():
            if os.environ.get("DT_NO_BUILD"):
                raise NativeError(f"runtime library {_build.RUNTIME_SO} missing or stale and DT_NO_BUILD is set")
            _build.build_runtime()
        L = ctypes.CDLL(_build.RUNTIME_SO)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name, None)
            if f is None:
                continue
            f.argtypes = args
            f.restype = res
        _RT = L
        return L


def register(name, argtypes, restype=c_int):
    f = getattr(rt(), name)
    f.argtypes = argtypes
    f.restype = restype
    return f


def last_error() -> str:
    e = rt().dtr_last_error()
    return e.decode() if e else ""


def take_blob(h) -> bytes:
    """Copy a runtime Blob into Python bytes and free it."""
    if not h:
        raise NativeError(last_error() or "native call failed")
    L = rt()
    try:
        n = L.dtr_blob_size(h)
        return ctypes.string_at(L.dtr_blob_data(h), n)
    finally:
        L.dtr_blob_free(h)


def zstd_compress(data: bytes, level: int = 3) -> bytes:
    return take_blob(rt().dtr_zstd_compress(data, len(data), level))


def zstd_decompress(data: bytes) -> bytes:
    return take_blob(rt().dtr_zstd_decompress(data, len(data)))


def shard_assignment(node_id: str, checkpoint_version: int, total_shards: int, shards_per_node: int):
    """Reference ``compute_shard_assignment`` (core/model/src/training.rs:229-270), bit-exact."""
    n = min(shards_per_node, total_shards)
    out = (ctypes.c_longlong * max(n, 1))()
    k = rt().dtr_shard_assignment(node_id.encode(), checkpoint_version, total_shards, shards_per_node, out)
    return [int(out[i]) for i in range(k)]
