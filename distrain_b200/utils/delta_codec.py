"""Delta wire formats.

* Reference format: zstd(JSON ``SparseDelta`` {indices, values, shapes, scales, config}), raw-JSON
  fallback without zstd, and detection of the low-rank JSON variant (compression.rs:92-104, 262-290,
  429-441; lowrank.rs:22-36; aggregation.rs:504-513). Encoding/decoding of the big arrays is native.
* DTZ1: this framework's binary format for a device payload (flat indices + int8 + per-block scales),
  what a node uploads when it talks to a coordinator outside its box.
"""
from __future__ import annotations

import ctypes
import json
from typing import Optional

import torch

from ..config import CompressionConfig
from .native import rt, take_blob, last_error, NativeError
from ..parallel.compression import SparseDeltaT


def encode_sparse_delta(sd: SparseDeltaT, zstd_level: int = 3) -> bytes:
    names = list(sd.shapes.keys())
    n = len(names)
    idx_t = [sd.indices.get(k, torch.zeros(0, dtype=torch.int64)).to(torch.int32).contiguous() for k in names]
    val_t = [sd.values.get(k, torch.zeros(0)).to(torch.float32).contiguous() for k in names]
    cnames = (ctypes.c_char_p * n)(*[k.encode() for k in names])
    ndims = (ctypes.c_int * n)(*[len(sd.shapes[k]) for k in names])
    dl = [int(s) for k in names for s in sd.shapes[k]]
    dims = (ctypes.c_longlong * max(len(dl), 1))(*dl)
    nk = (ctypes.c_longlong * n)(*[t.numel() for t in idx_t])
    ip = (ctypes.c_void_p * n)(*[t.data_ptr() for t in idx_t])
    vp = (ctypes.c_void_p * n)(*[t.data_ptr() for t in val_t])
    sc = None
    if sd.scales is not None:
        sc = (ctypes.c_float * n)(*[float(sd.scales.get(k, 1.0)) for k in names])
    cfg = json.dumps(sd.config.reference_dict() if isinstance(sd.config, CompressionConfig) else sd.config).encode()
    h = rt().dtr_sparse_delta_encode(n, cnames, ndims, dims, nk, ip, vp, sc, cfg, zstd_level)
    return take_blob(h)


class LowRankPayload(dict):
    """Parsed low-rank delta JSON ({"tensors": {name: {u, v, m, n, rank}}, "rank": r})."""


def decode_delta(data: bytes):
    """zstd / raw JSON -> {name: dense fp32 tensor (flat)}; a low-rank payload is returned as LowRankPayload."""
    L = rt()
    buf = ctypes.create_string_buffer(bytes(data), len(data))
    h = L.dtr_delta_decode(buf, len(data))
    if not h:
        raise NativeError(last_error())
    try:
        if L.dtr_delta_is_lowrank(h):
            return LowRankPayload(json.loads(L.dtr_delta_raw_json(h).decode()))
        out = {}
        for i in range(L.dtr_delta_count(h)):
            name = L.dtr_delta_name(h, i).decode()
            n = L.dtr_delta_numel(h, i)
            t = torch.empty(n, dtype=torch.float32)
            ctypes.memmove(t.data_ptr(), L.dtr_delta_data(h, i), n * 4)
            out[name] = t
        return out
    finally:
        L.dtr_delta_free(h)


def encode_dtz(total_params: int, idx: torch.Tensor, q: Optional[torch.Tensor], scales: Optional[torch.Tensor],
               values: Optional[torch.Tensor], block: int, zstd_level: int = 0) -> bytes:
    idx = idx.to(torch.int32).cpu().contiguous()
    count = idx.numel()
    qp = q.cpu().contiguous() if q is not None else None
    sp = scales.cpu().contiguous() if scales is not None else None
    vp = values.cpu().contiguous() if values is not None else None
    h = rt().dtr_dtz_encode(total_params, count, idx.data_ptr(), qp.data_ptr() if qp is not None else None,
                            sp.data_ptr() if sp is not None else None, vp.data_ptr() if vp is not None else None,
                            block, zstd_level)
    return take_blob(h)


def decode_dtz_dense(data: bytes) -> torch.Tensor:
    buf = ctypes.create_string_buffer(bytes(data), len(data))
    raw = take_blob(rt().dtr_dtz_decode_dense(buf, len(data)))
    return torch.frombuffer(bytearray(raw), dtype=torch.float32)


def payload_to_sparse_delta(payload, count: int, layout, cfg: CompressionConfig) -> SparseDeltaT:
    """Device payload -> reference SparseDelta (per-tensor indices; dequantised values)."""
    idx = payload.global_indices(count).cpu()
    if payload.block:
        q = payload.q[:count].float().cpu()
        sc = payload.scales[:(count + payload.block - 1) // payload.block].cpu()
        vals = q * sc[torch.arange(count) // payload.block]
    else:
        vals = payload.val[:count].cpu()
    indices, values, shapes = {}, {}, {}
    for e in layout.entries:
        lo = torch.searchsorted(idx, e.offset)
        hi = torch.searchsorted(idx, e.offset + e.numel)
        indices[e.name] = idx[lo:hi] - e.offset
        values[e.name] = vals[lo:hi]
        shapes[e.name] = list(e.shape)
    return SparseDeltaT(indices=indices, values=values, shapes=shapes, scales=None, config=cfg)
