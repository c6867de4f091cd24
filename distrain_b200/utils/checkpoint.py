"""Checkpoint I/O: safetensors (reference core/model/src/checkpoint.rs) through the C++ runtime.

Reads F32 / BF16 / F16 tensors as fp32, writes F32, in the reference's PyTorch ``[out, in]`` layout with
its state-dict names (model.rs:401-467). The optimizer velocity file uses the ``velocity.`` prefix and
flat shapes (aggregation.rs:391-408).
"""
from __future__ import annotations

import ctypes
import json
from typing import Dict, Optional

import torch

from .native import rt, take_blob, last_error, NativeError


def _read(h) -> Dict[str, torch.Tensor]:
    L = rt()
    out = {}
    try:
        for i in range(L.dtr_st_count(h)):
            name = L.dtr_st_name(h, i).decode()
            shape = [L.dtr_st_dim(h, i, d) for d in range(L.dtr_st_ndim(h, i))]
            numel = 1
            for s in shape:
                numel *= s
            t = torch.empty(numel, dtype=torch.float32)
            n = L.dtr_st_read_f32(h, i, t.data_ptr(), numel)
            if n < 0:
                raise NativeError(last_error())
            out[name] = t.view(shape) if shape else t.view(())
    finally:
        L.dtr_st_close(h)
    return out


def load_safetensors(path: str) -> Dict[str, torch.Tensor]:
    h = rt().dtr_st_open(path.encode())
    if not h:
        raise NativeError(last_error())
    return _read(h)


def load_safetensors_bytes(data: bytes) -> Dict[str, torch.Tensor]:
    buf = ctypes.create_string_buffer(data, len(data))
    h = rt().dtr_st_open_bytes(buf, len(data))
    if not h:
        raise NativeError(last_error())
    return _read(h)


def _save_args(tensors: Dict[str, torch.Tensor]):
    names = list(tensors.keys())
    conts = [tensors[n].detach().to("cpu", torch.float32).contiguous() for n in names]
    cnames = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
    ndims = (ctypes.c_int * len(names))(*[t.dim() for t in conts])
    dims_list = [s for t in conts for s in t.shape]
    dims = (ctypes.c_longlong * max(len(dims_list), 1))(*dims_list)
    ptrs = (ctypes.c_void_p * len(names))(*[t.data_ptr() for t in conts])
    return names, conts, cnames, ndims, dims, ptrs


def save_safetensors(tensors: Dict[str, torch.Tensor], path: Optional[str] = None,
                     metadata: Optional[Dict[str, str]] = None) -> Optional[bytes]:
    """Write fp32 safetensors to ``path`` (atomic rename); with path None return the bytes."""
    names, conts, cnames, ndims, dims, ptrs = _save_args(tensors)
    meta = json.dumps(metadata).encode() if metadata else None
    if path is not None:
        rc = rt().dtr_st_save(path.encode(), len(names), cnames, ndims, dims, ptrs, meta, None)
        if rc:
            raise NativeError(last_error())
        return None
    blob = ctypes.c_void_p()
    rc = rt().dtr_st_save(None, len(names), cnames, ndims, dims, ptrs, meta, ctypes.byref(blob))
    if rc:
        raise NativeError(last_error())
    return take_blob(blob.value)


def save_velocity(velocity: Dict[str, torch.Tensor], path: Optional[str] = None):
    """Velocity file: ``velocity.<name>`` keys with flat shapes (aggregation.rs:391-408)."""
    return save_safetensors({f"velocity.{k}": v.reshape(-1) for k, v in velocity.items()}, path)


def load_velocity(path_or_bytes) -> Dict[str, torch.Tensor]:
    sd = load_safetensors_bytes(path_or_bytes) if isinstance(path_or_bytes, (bytes, bytearray)) else \
        load_safetensors(path_or_bytes)
    return {k[len("velocity."):]: v for k, v in sd.items() if k.startswith("velocity.")}
