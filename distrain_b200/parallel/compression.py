"""Delta compression: error feedback -> (adaptive) top-k -> INT8 -> payload.

Two implementations of the same algorithm (reference core/model/src/compression.rs:57-382):

* ``DeviceCompressor`` - the node's hot path: the fused sm_100a pipeline in ``csrc/kernels/compress.cu``
  over the flat parameter buffer. ``begin()`` (on the training stream) forms d = snapshot - master + ef
  and re-snapshots; ``finish()`` (on a side stream) selects, compacts, quantises and leaves a payload
  (ascending flat indices, int8 values, fp32 per-block scales) in device memory.
* ``compress_reference`` - a CPU restatement over a name->tensor dict, the oracle for tests and the
  CPU node path; its output is the reference's ``SparseDelta`` (JSON/zstd codec in
  ``utils/delta_codec.py``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from ..config import CompressionConfig


# ─────────────────────────────── CPU reference ───────────────────────────────
def sparsify_topk(delta: Dict[str, torch.Tensor], k_fraction: float, adaptive: bool):
    """Returns (sparse dense-shaped, indices, values) per tensor (compression.rs:128-184).
    Ties are broken by ascending index (stable sort by |value| descending)."""
    names = list(delta.keys())
    norms = {n: math.sqrt(float((delta[n].double() ** 2).sum())) for n in names} if adaptive else {}
    total_norm = sum(norms.values())
    total_params = sum(delta[n].numel() for n in names)
    kf32 = float(torch.tensor(k_fraction, dtype=torch.float32))
    total_budget = math.ceil(total_params * kf32)
    sparse, idxs, vals = {}, {}, {}
    for n in names:
        flat = delta[n].reshape(-1).float()
        L = flat.numel()
        if adaptive and total_norm > 0:
            k = math.ceil(total_budget * (norms[n] / total_norm))
            k = min(max(k, 1), L)
        else:
            k = max(int(math.ceil(float(torch.tensor(L, dtype=torch.float32) * torch.tensor(k_fraction,
                                                                                            dtype=torch.float32)))), 1)
            k = min(k, L)
        order = torch.sort(flat.abs(), descending=True, stable=True).indices[:k]
        order = torch.sort(order).values
        v = flat[order]
        sp = torch.zeros_like(flat)
        sp[order] = v
        sparse[n] = sp
        idxs[n] = order.to(torch.int64)
        vals[n] = v
    return sparse, idxs, vals


def quantize_int8(values: torch.Tensor, block: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """absmax/127 scale per block (block 0 = one scale for the whole vector), round half away from 0."""
    v = values.float().reshape(-1)
    n = v.numel()
    if block <= 0:
        block = max(n, 1)
    nb = max((n + block - 1) // block, 1)
    pad = nb * block - n
    vp = torch.cat([v, v.new_zeros(pad)]) if pad else v
    vb = vp.view(nb, block)
    amax = vb.abs().amax(dim=1)
    scale = torch.where(amax == 0, torch.ones_like(amax), amax / 127.0)
    r = vb / scale[:, None]
    q = torch.sign(r) * torch.floor(r.abs() + 0.5)
    q = q.clamp(-127, 127).to(torch.int8).reshape(-1)[:n]
    return q, scale


def dequantize_int8(q: torch.Tensor, scale: torch.Tensor, block: int = 0) -> torch.Tensor:
    n = q.numel()
    if block <= 0:
        block = max(n, 1)
    idx = torch.arange(n) // block
    return q.float() * scale[idx]


@dataclass
class SparseDeltaT:
    """In-memory SparseDelta (compression.rs:92-104) with tensors instead of JSON lists."""
    indices: Dict[str, torch.Tensor]
    values: Dict[str, torch.Tensor]      # dequantised fp32 values, as the reference stores them
    shapes: Dict[str, List[int]]
    scales: Optional[Dict[str, float]]
    config: CompressionConfig


def compress_reference(delta: Dict[str, torch.Tensor], shapes: Dict[str, List[int]], cfg: CompressionConfig,
                       ef: Dict[str, torch.Tensor]):
    """Error feedback -> top-k -> per-tensor INT8 (reference semantics). Updates ``ef`` in place.
    Returns (SparseDeltaT, stats dict)."""
    combined = {n: delta[n].reshape(-1).float() + (ef[n].reshape(-1) if n in ef else 0) for n in delta}
    dense_norm = math.sqrt(sum(float((t.double() ** 2).sum()) for t in combined.values()))
    sparse, idxs, vals = sparsify_topk(combined, cfg.top_k_fraction, cfg.per_tensor_adaptive)
    for n in combined:
        ef[n] = combined[n] - sparse[n]
    sparse_norm = math.sqrt(sum(float((t.double() ** 2).sum()) for t in sparse.values()))
    kept = sum(int((t != 0).sum()) for t in sparse.values())
    scales = None
    if cfg.quantize_int8:
        scales = {}
        for n in vals:
            q, s = quantize_int8(vals[n], 0)
            vals[n] = dequantize_int8(q, s, 0)
            scales[n] = float(s[0])
    sd = SparseDeltaT(indices=idxs, values=vals, shapes=shapes, scales=scales, config=cfg)
    total = sum(t.numel() for t in combined.values())
    stats = {"dense_norm": dense_norm, "sparse_norm": sparse_norm,
             "retention_ratio": sparse_norm / dense_norm if dense_norm > 0 else 0.0,
             "top_k_fraction": cfg.top_k_fraction, "num_params_total": total, "num_params_kept": kept,
             "raw_param_bytes": total * 4}
    return sd, stats


def reconstruct_dense(sd: SparseDeltaT) -> Dict[str, torch.Tensor]:
    out = {}
    for n, shape in sd.shapes.items():
        numel = 1
        for s in shape:
            numel *= s
        flat = torch.zeros(numel)
        if n in sd.indices and sd.indices[n].numel():
            flat[sd.indices[n].long()] = sd.values[n].float()
        out[n] = flat
    return out


def adaptive_top_k(loss: float, max_delta_bytes: Optional[int], raw_param_bytes: int) -> float:
    """Loss-based retention, capped by the bandwidth budget (reference trainer.rs:33-70)."""
    if loss > 20.0:
        k = 0.50
    elif loss > 10.0:
        k = 0.60
    elif loss > 7.0:
        k = 0.70
    elif loss > 5.0:
        k = 0.75
    else:
        k = 0.80
    if max_delta_bytes is not None:
        mx = max_delta_bytes / (raw_param_bytes * 0.5) if raw_param_bytes > 0 else k
        k = max(min(k, mx), 0.01)
    return k


def adaptive_push_mode(bandwidth_adaptive: bool, bandwidth_bps: float, raw_bytes: int, last_loss: float,
                       cfg: CompressionConfig):
    """(kind, top-k fraction, int8 block) of a push (reference continuous.rs:190-219): without the
    bandwidth-adaptive policy, the configured top-k; with it and no measured bandwidth, the loss-based
    top-k (quantised as configured); with a bandwidth under which the raw delta moves within the 10 s
    budget, raw (dense fp32); otherwise an unquantised top-k capped by that budget."""
    qb = cfg.int8_block if cfg.quantize_int8 else 0
    if not bandwidth_adaptive:
        return "topk", cfg.top_k_fraction, qb
    if bandwidth_bps <= 0.0:
        return "topk", adaptive_top_k(last_loss, None, 0), qb
    budget = bandwidth_bps * 10.0
    if raw_bytes <= budget:
        return "raw", 1.0, 0
    return "topk", adaptive_top_k(last_loss, int(budget), raw_bytes), 0


# ─────────────────────────────── device pipeline ───────────────────────────────
class DeviceCompressor:
    """Fused compress pipeline over a ``ParamLayout``'s flat buffer (one per node)."""

    def __init__(self, layout, device, cfg: CompressionConfig, payload=None):
        from ..ops import _lib
        from ..ops._lib import c_int, c_void, c_ll, c_float
        self.L = _lib.lib()
        _lib.register("dt_compress_workspace_bytes", [c_int, c_int], restype=c_ll)
        _lib.register("dt_compress_begin", [c_void, c_void, c_void, c_void, c_void, c_void, c_int, c_int, c_void,
                                            c_void, c_int, c_void])
        _lib.register("dt_compress_finish", [c_void, c_void, c_void, c_void, c_int, c_int, c_void, c_float, c_int,
                                             c_void, c_void, c_void, c_void, c_int, c_ll, c_void, c_int, c_void,
                                             c_void])
        _lib.register("dt_compress_export_stats", [c_void, c_int, c_int, c_void, c_void])
        _lib.register("dt_compress_raw", [c_void, c_void, c_ll, c_void])
        _lib.register("dt_compress_stats_len", [c_int], restype=c_ll)
        self.layout, self.device, self.cfg = layout, torch.device(device), cfg
        n = layout.total
        self.cseg, self.cstart, self.cend, self.nseg = layout.chunk_tables(self.device)
        self.nchunks = self.cseg.numel()
        # first chunk of every 2^31-element index window (kept indices are stored window-relative)
        W = layout.WINDOW
        self.nwin = max(1, (layout.total + W - 1) // W)
        starts = self.cstart.cpu()
        win_chunk = [0] + [int(torch.searchsorted(starts, k * W)) for k in range(1, self.nwin)]
        self.win_chunk = torch.tensor(win_chunk, dtype=torch.int32, device=self.device)
        self.seg_len = torch.tensor([e.numel for e in layout.entries], dtype=torch.int64, device=self.device)
        self.snap = torch.zeros(n, dtype=torch.float32, device=self.device)
        self.ef = torch.zeros(n, dtype=torch.float32, device=self.device)
        wsb = self.L.dt_compress_workspace_bytes(self.nseg, self.nchunks)
        self.ws = torch.zeros(wsb, dtype=torch.uint8, device=self.device)
        nstat = self.L.dt_compress_stats_len(self.nseg)  # doubles dt_compress_export_stats writes
        self.stats_dev = torch.zeros(nstat, dtype=torch.float64, device=self.device)
        self.stats_host = torch.zeros(nstat, dtype=torch.float64).pin_memory()
        self.capacity = self.capacity_for(layout, cfg.top_k_fraction)
        self.payload = payload or DevicePayload.allocate(self.capacity, cfg.int8_block if cfg.quantize_int8 else 0,
                                                         self.device)

    @staticmethod
    def capacity_for(layout, k_fraction: float) -> int:
        total = layout.num_params()
        cap = math.ceil(total * float(k_fraction)) + len(layout.entries) + 16
        return min(cap, total)

    def reset(self, master: torch.Tensor):
        """New checkpoint: snapshot <- master, error feedback cleared."""
        self.snap.copy_(master)
        self.ef.zero_()

    def begin(self, master: torch.Tensor, stream=None):
        from ..ops._lib import check, stream_ptr
        check(self.L.dt_compress_begin(master.data_ptr(), self.snap.data_ptr(), self.ef.data_ptr(),
                                       self.cseg.data_ptr(), self.cstart.data_ptr(), self.cend.data_ptr(),
                                       self.nchunks, self.nseg, self.seg_len.data_ptr(), self.ws.data_ptr(), 1,
                                       stream_ptr(stream)), "dt_compress_begin")

    def finish(self, payload=None, stream=None, k_fraction: Optional[float] = None,
               quant_block: Optional[int] = None):
        """Selection, compaction and (quant_block > 0) INT8 quantisation into ``payload``; ``k_fraction`` and
        ``quant_block`` default to the configuration (quant_block 0: fp32 values, the payload's q and
        scales untouched)."""
        from ..ops._lib import check, stream_ptr
        p = payload or self.payload
        kf = self.cfg.top_k_fraction if k_fraction is None else k_fraction
        qb = (self.cfg.int8_block if self.cfg.quantize_int8 else 0) if quant_block is None else quant_block
        assert qb == 0 or p.block == qb, "payload laid out for another quantisation block"
        assert math.ceil(self.layout.num_params() * kf) <= p.capacity or kf >= 1.0, "payload capacity"
        check(self.L.dt_compress_finish(self.ef.data_ptr(), self.cseg.data_ptr(), self.cstart.data_ptr(),
                                        self.cend.data_ptr(), self.nchunks, self.nseg, self.ws.data_ptr(), float(kf),
                                        int(self.cfg.per_tensor_adaptive), p.idx.data_ptr(), p.val.data_ptr(),
                                        p.q.data_ptr() if qb else None, p.scales.data_ptr() if qb else None, qb,
                                        p.capacity, self.win_chunk.data_ptr(), self.nwin, p.win.data_ptr(),
                                        stream_ptr(stream)), "dt_compress_finish")
        check(self.L.dt_compress_export_stats(self.ws.data_ptr(), self.nseg, self.nchunks, self.stats_dev.data_ptr(),
                                              stream_ptr(stream)), "dt_compress_export_stats")
        with torch.cuda.stream(stream if stream is not None else torch.cuda.current_stream()):
            self.stats_host.copy_(self.stats_dev, non_blocking=True)

    def finish_raw(self, out: torch.Tensor, stream=None):
        """Raw push after ``begin``: the dense delta (+ error feedback) into ``out`` (fp32, >= n elements),
        error feedback cleared. Statistics as for a top-k push (``read_stats(raw=True)``)."""
        from ..ops._lib import check, stream_ptr
        n = self.layout.total
        assert out.dtype == torch.float32 and out.numel() >= n
        check(self.L.dt_compress_export_stats(self.ws.data_ptr(), self.nseg, self.nchunks, self.stats_dev.data_ptr(),
                                              stream_ptr(stream)), "dt_compress_export_stats")
        check(self.L.dt_compress_raw(self.ef.data_ptr(), out.data_ptr(), n, stream_ptr(stream)), "dt_compress_raw")
        with torch.cuda.stream(stream if stream is not None else torch.cuda.current_stream()):
            self.stats_host.copy_(self.stats_dev, non_blocking=True)

    def read_stats(self, raw: bool = False, quantized: Optional[bool] = None) -> dict:
        """Call after the finish stream has been synchronised. ``wire`` = [sum of squares, max |x|,
        non-finite count] of the values exactly as they were sent (dequantised for INT8 pushes, the kept
        fp32 values for unquantised ones, the whole delta for raw ones): what the coordinator validates
        and clips on."""
        s = self.stats_host
        ns = self.nseg
        seg = s[:ns * 6].view(ns, 6)
        total_kept = int(s[ns * 6].item())
        dense_sq, kept_sq = float(seg[:, 0].sum()), float(seg[:, 1].sum())
        max_abs, nonfinite = float(seg[:, 3].max()), float(seg[:, 4].sum())
        if raw:
            total_kept, kept_sq = self.layout.total, dense_sq
        if quantized is None:
            quantized = self.cfg.quantize_int8
        if quantized and not raw:
            wire = [float(s[ns * 6 + 1]), float(s[ns * 6 + 2]), float(s[ns * 6 + 3]) + nonfinite]
        else:  # the largest |d| of a tensor is always kept, so max |kept| = max |d|
            wire = [kept_sq, max_abs, nonfinite]
        dense_norm, sparse_norm = math.sqrt(dense_sq), math.sqrt(kept_sq)
        return {"dense_norm": dense_norm, "sparse_norm": sparse_norm,
                "retention_ratio": sparse_norm / dense_norm if dense_norm > 0 else 0.0,
                "num_params_total": self.layout.num_params(), "num_params_kept": total_kept,
                "max_abs": max_abs, "nonfinite": nonfinite > 0, "wire": wire,
                "k_per_tensor": seg[:, 2].long().tolist()}


class DevicePayload:
    """Compressed delta in device memory: idx int32[cap], val fp32[cap], q int8[cap], scales fp32[cap/blk],
    win int64[8]. Views into one allocation so the whole payload can live in a single symmetric (peer-mapped)
    buffer. ``idx`` holds each kept index relative to its 2^31-element window; ``win[k]`` is the position
    of the first entry of window k (int64 max for windows that do not exist), so the flat index of entry
    p is idx[p] + (k << 31) with k the number of window starts <= p beyond the first."""

    MAX_WINDOWS = 8

    def __init__(self, buf: torch.Tensor, capacity: int, block: int):
        self.buf, self.capacity, self.block = buf, capacity, block
        o = 0
        def take(nbytes):
            nonlocal o
            s = o
            o = (o + nbytes + 255) // 256 * 256
            return s
        oi = take(4 * capacity)
        ov = take(4 * capacity)
        oq = take(capacity)
        nb = (capacity + block - 1) // block if block else 1
        os_ = take(4 * nb)
        ow = take(8 * self.MAX_WINDOWS)
        self.win = buf[ow:ow + 8 * self.MAX_WINDOWS].view(torch.int64)
        self.idx = buf[oi:oi + 4 * capacity].view(torch.int32)
        self.val = buf[ov:ov + 4 * capacity].view(torch.float32)
        self.q = buf[oq:oq + capacity].view(torch.int8)
        self.scales = buf[os_:os_ + 4 * nb].view(torch.float32)

    @staticmethod
    def nbytes(capacity: int, block: int) -> int:
        nb = (capacity + block - 1) // block if block else 1
        r = lambda x: (x + 255) // 256 * 256
        return r(4 * capacity) + r(4 * capacity) + r(capacity) + r(4 * nb) + r(8 * DevicePayload.MAX_WINDOWS)

    def global_indices(self, count: int) -> torch.Tensor:
        """Flat int64 indices of the first ``count`` kept entries."""
        pos = torch.arange(count, device=self.idx.device, dtype=torch.int64)
        k = torch.zeros_like(pos)
        for w in self.win[1:].tolist():
            k += (pos >= w).long()
        return self.idx[:count].long() + (k << 31)

    @classmethod
    def allocate(cls, capacity: int, block: int, device) -> "DevicePayload":
        buf = torch.zeros(cls.nbytes(capacity, block), dtype=torch.uint8, device=device)
        return cls(buf, capacity, block)

    def wire_bytes(self, count: int, block: Optional[int] = None) -> int:
        """Bytes a contribution of `count` kept entries occupies on the wire (idx + int8/fp32 + scales);
        `block` overrides the payload's quantisation block (0: fp32 values)."""
        blk = self.block if block is None else block
        if blk:
            return count * 4 + count + ((count + blk - 1) // blk) * 4
        return count * 8

    def raw(self, n: int) -> torch.Tensor:
        """The slot read as a dense fp32 delta of n values (a raw push; the slot must hold 4n bytes)."""
        assert self.buf.numel() >= 4 * n, "payload slot too small for a raw push"
        return self.buf[:4 * n].view(torch.float32)
