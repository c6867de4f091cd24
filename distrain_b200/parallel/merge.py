"""Coordinator merge: validate -> 3x running-average norm clip -> staleness x tokens weighted average ->
outer (Nesterov) apply, reference coordinator/src/aggregation.rs:154-472.

* ``merge_reference`` - CPU restatement over name->tensor dicts (oracle; also the CPU coordinator path).
* ``DeviceMerger``   - the in-box path: contributions are compressed payloads that stay in each node's
  GPU memory; the sm_100a kernels in ``csrc/kernels/merge.cu`` read them through peer pointers,
  dequantise, weight and scatter-add into a local fp32 accumulator, then apply the update to the global
  checkpoint and write it (fp32 + bf16) into every node's staging buffer in the same pass.
"""
from __future__ import annotations

import ctypes
import os
import math
import struct
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from ..protocol import clip_scales, validate_stats


# ─────────────────────────────── CPU reference ───────────────────────────────
def validate_delta(delta: Dict[str, torch.Tensor]) -> Optional[str]:
    if not delta:
        return "Empty delta"
    sumsq = 0.0
    for name, v in delta.items():
        v = v.float()
        if torch.isnan(v).any():
            return f"NaN in {name}"
        if torch.isinf(v).any():
            return f"Inf in {name}"
        mx = float(v.abs().max()) if v.numel() else 0.0
        if mx > 100.0:
            return f"Magnitude too large in {name}: {mx:.1f}"
        sumsq += float((v.double() ** 2).sum())
    n = math.sqrt(sumsq)
    if n > 1000.0:
        return f"Total norm too large: {n:.1f}"
    if n < 1e-10:
        return f"Total norm near zero: {n:.2e}"
    return None


def weighted_average(deltas: Sequence[Tuple[Dict[str, torch.Tensor], float]]):
    if not deltas:
        return None
    tot = sum(w for _, w in deltas)
    if tot == 0:
        return None
    keys = list(deltas[0][0].keys())
    out = {}
    for k in keys:
        acc = torch.zeros_like(deltas[0][0][k], dtype=torch.float32)
        for d, w in deltas:
            if k in d:
                acc = acc + d[k].float() * float(w / tot)
        out[k] = acc
    return out


def nesterov_step(ckpt: Dict[str, torch.Tensor], avg: Dict[str, torch.Tensor], velocity: Optional[Dict], lr: float,
                  mu: float):
    if velocity is None:
        velocity = {k: torch.zeros_like(v) for k, v in avg.items()}
    for k, p in ckpt.items():
        if k in avg:
            v = velocity[k] * mu + avg[k]
            velocity[k] = v
            ckpt[k] = p - (v * mu + avg[k]) * lr
    return ckpt, velocity


def merge_reference(ckpt: Dict[str, torch.Tensor], deltas: List[Dict[str, torch.Tensor]], weights: List[float],
                    velocity=None, outer_lr: float = 1.0, outer_momentum: float = 0.0):
    """Returns (new_ckpt, velocity, info). Order of ``deltas`` = arrival order (matters for clipping)."""
    accepted, norms, rejected = [], [], 0
    eff = []
    for d, w in zip(deltas, weights):
        if validate_delta(d) is not None:
            rejected += 1
            continue
        n = math.sqrt(sum(float((t.double() ** 2).sum()) for t in d.values()))
        e = n
        if eff:
            avg = sum(eff) / len(eff)
            mx = avg * 3.0
            if n > mx and n > 0:
                s = mx / n
                d = {k: t * s for k, t in d.items()}
                e = mx
        eff.append(e)
        accepted.append((d, w))
    avg = weighted_average(accepted)
    if avg is None:
        raise RuntimeError("No valid deltas to aggregate")
    delta_norm = math.sqrt(sum(float((t.double() ** 2).sum()) for t in avg.values()))
    new = {k: v.clone() for k, v in ckpt.items()}
    new, velocity = nesterov_step(new, avg, velocity, outer_lr, outer_momentum)
    return new, velocity, {"accepted": len(accepted), "rejected": rejected, "outer_delta_norm": delta_norm,
                           "per_delta_norms": eff}


# ─────────────────────────────── device merge ───────────────────────────────
@dataclass
class Contribution:
    """One payload resident in (possibly another GPU's) device memory."""
    idx_ptr: int
    q_ptr: int
    val_ptr: int
    scales_ptr: int
    count: int
    block: int
    dense: bool
    weight: float
    node_id: str = ""
    wire_bytes: int = 0
    win_ptr: int = 0  # the payload's window starts (DevicePayload.win), 0 = one window


_CONTRIB_FMT = "<QQQQQqiifi"  # matches struct Contrib in merge.cu (64 bytes)
DT_WAIT_SHORT_NS = 2_000_000_000  # device-side checks that the host protocol has already satisfied


class DeviceMerger:
    """Device merge of compressed payloads into the global checkpoint ``theta``.

    ``theta_buffer``: an fp32 [n] tensor that holds the checkpoint and is updated in place (the in-box
    coordinator passes its own staging buffer, so the checkpoint exists once on that GPU); it is
    initialised from ``theta_init`` when that is given too. Without ``theta_buffer`` theta is a copy of
    ``theta_init``. With ``momentum`` 0 (the reference's outer step, coordinator/src/aggregation.rs:364)
    the weighted dequantised values are scatter-added straight into theta; otherwise through an fp32
    accumulator and a velocity buffer (Nesterov, aggregation.rs:64-105)."""

    def __init__(self, n_params_padded: int, device, theta_init: Optional[torch.Tensor] = None,
                 momentum: float = 0.0, stream: Optional[torch.cuda.Stream] = None,
                 theta_buffer: Optional[torch.Tensor] = None):
        from ..ops import _lib
        from ..ops._lib import c_int, c_void, c_ll, c_float
        self.L = _lib.lib()
        _lib.register("dt_merge_contrib_bytes", [], restype=c_ll)
        _lib.register("dt_merge_prepass", [c_void, c_int, c_ll, c_void, c_void])
        _lib.register("dt_merge_accumulate", [c_void, c_int, c_ll, c_void, c_void])
        _lib.register("dt_merge_apply_broadcast", [c_void, c_void, c_void, c_ll, c_float, c_float, c_void, c_void,
                                                   c_int, c_void])
        _lib.register("dt_merge_broadcast", [c_void, c_ll, c_void, c_void, c_int, c_void])
        assert self.L.dt_merge_contrib_bytes() == struct.calcsize(_CONTRIB_FMT)
        self.device = torch.device(device)
        self.n = n_params_padded
        if theta_buffer is not None:
            assert theta_buffer.dtype == torch.float32 and theta_buffer.numel() == self.n
            self.theta = theta_buffer
            if theta_init is not None:
                self.theta.copy_(theta_init)
        else:
            self.theta = theta_init.to(self.device, torch.float32).clone()
        self.momentum = float(momentum)
        self.acc = torch.zeros(self.n, dtype=torch.float32, device=self.device) if momentum else None
        self.vel = torch.zeros(self.n, dtype=torch.float32, device=self.device) if momentum else None
        self.stream = stream or torch.cuda.Stream(device=self.device, priority=0)
        self.stats = torch.zeros(3 * 64, dtype=torch.float64, device=self.device)
        self.stats_host = torch.zeros(3 * 64, dtype=torch.float64).pin_memory()

    def _pack(self, contribs: List[Contribution], coefs: List[float]):
        """Host descriptor table (struct Contrib records), passed to the kernels as launch parameters."""
        import ctypes
        fmt = _CONTRIB_FMT
        raw = b"".join(struct.pack(fmt, c.idx_ptr if not c.dense else 0, c.q_ptr, c.val_ptr, c.scales_ptr,
                                   c.win_ptr if not c.dense else 0, c.count, max(c.block, 1), int(c.dense), float(k),
                                   0) for c, k in zip(contribs, coefs))
        buf = ctypes.create_string_buffer(raw, len(raw))
        self._keep = buf
        return buf

    def _prepass(self, contribs: List[Contribution], maxc: int):
        from ..ops._lib import check
        st = self.stream
        n = len(contribs)
        buf = self._pack(contribs, [1.0] * n)
        with torch.cuda.stream(st):
            check(self.L.dt_merge_prepass(buf, n, maxc, self.stats.data_ptr(), st.cuda_stream), "dt_merge_prepass")
            self.stats_host[:3 * n].copy_(self.stats[:3 * n], non_blocking=True)
        st.synchronize()
        return self.stats_host[:3 * n].view(n, 3).tolist()

    def prepass(self, contribs: List[Contribution]) -> List[List[float]]:
        """Per-contribution [sum of squares, max |x|, non-finite flag] of the dequantised payloads; blocks the
        calling (coordinator) thread until they are on the host."""
        n = len(contribs)
        assert 0 < n <= 64
        return self._prepass(contribs, max(c.count for c in contribs))

    @staticmethod
    def plan(contribs: List[Contribution], stats: List[List[float]]):
        """Validation, norm clipping in arrival order and weighting from (possibly shard-combined) stats:
        returns (coefficient per contribution, info). Raises when no contribution is valid."""
        n = len(contribs)
        valid, norms, reasons = [], [], []
        for i, (sumsq, mx, nf) in enumerate(stats):
            r = validate_stats(sumsq, mx, nf > 0, empty=contribs[i].count == 0)
            reasons.append(r)
            if r is None:
                valid.append(i)
                norms.append(math.sqrt(sumsq))
        if not valid:
            raise RuntimeError("No valid deltas to aggregate: " + "; ".join(str(r) for r in reasons))
        scales, eff = clip_scales(norms)
        wsum = sum(contribs[i].weight for i in valid)
        coefs = [0.0] * n
        for j, i in enumerate(valid):
            coefs[i] = contribs[i].weight / wsum * scales[j]
        return coefs, {"accepted": len(valid), "rejected": n - len(valid), "reasons": reasons,
                       "per_delta_norms": eff, "coefs": coefs}

    def accumulate_apply(self, contribs: List[Contribution], coefs: List[float], outer_lr: float,
                         mc32: int = 0, stage32: Sequence[int] = ()):
        """Weighted dequant scatter-add of every payload into the checkpoint, then the broadcast of the new
        checkpoint (multicast address ``mc32``, or the peers' staging pointers ``stage32``), enqueued on the
        merge stream."""
        from ..ops._lib import check
        import ctypes
        n = len(contribs)
        st = self.stream
        sp = st.cuda_stream
        maxc = max(c.count for c in contribs)
        s32 = (ctypes.c_void_p * max(len(stage32), 1))(*stage32) if stage32 else None
        with torch.cuda.stream(st):
            if self.acc is None:  # theta -= lr * sum_c coef_c * x_c, in place
                buf = self._pack(contribs, [-float(outer_lr) * k for k in coefs])
                check(self.L.dt_merge_accumulate(buf, n, maxc, self.theta.data_ptr(), sp), "dt_merge_accumulate")
                check(self.L.dt_merge_broadcast(self.theta.data_ptr(), self.n, mc32 or None, s32, len(stage32), sp),
                      "dt_merge_broadcast")
            else:
                buf = self._pack(contribs, coefs)
                check(self.L.dt_merge_accumulate(buf, n, maxc, self.acc.data_ptr(), sp), "dt_merge_accumulate")
                check(self.L.dt_merge_apply_broadcast(self.theta.data_ptr(), self.vel.data_ptr(), self.acc.data_ptr(),
                                                      self.n, float(outer_lr), self.momentum, mc32 or None, s32,
                                                      len(stage32), sp), "dt_merge_apply_broadcast")

    def merge(self, contribs: List[Contribution], outer_lr: float, mc32: int = 0, stage32: Sequence[int] = ()):
        """Full merge on ``self.stream``; blocks the calling (coordinator) thread on the prepass only.
        Returns an info dict (accepted, rejected, norms, nvlink bytes)."""
        n = len(contribs)
        coefs, info = self.plan(contribs, self.prepass(contribs))
        self.accumulate_apply(contribs, coefs, outer_lr, mc32, stage32)
        info["pulled_bytes"] = sum(contribs[i].wire_bytes for i in range(n))
        return info


class DistributedMerger:
    """This node's part of the distributed merge (merge.cu ``dm_*`` kernels): node r of W owns the flat
    range [a_r, b_r) of the checkpoint. Rank 0 plans an attempt on the host from the statistics each node
    reported with its push (``DeviceMerger.plan``: validation, clipping, weights) and announces members and
    coefficients; every node then pulls its range of each member payload over NVLink, adds it into its
    slice of the checkpoint in its own staging slot and writes the slice into every node's slot, through
    NVLS multicast or per-peer stores (``apply``); rank 0 checks that all slices landed (``finish``).
    Every payload is read once, by the node that owns the slice, and the broadcast is spread over all W
    GPUs instead of funnelling through one. The caller orders the steps across nodes (announcement
    before ``apply``, every node's completion before ``finish``), so no kernel waits on another node's
    host progress.

    ``ctl``: this node's control buffer (``CTL_BYTES``, symmetric), ``ctl_ptrs``: every node's control
    buffer by rank; ``theta``: this node's fp32 staging slot (all slots hold the same checkpoint between
    merges); ``stage_ptrs`` / ``stage_mc``: every node's slot, and the multicast address (0 = none)."""

    CTL_BYTES = 8192
    OFF_COEF, OFF_DONE, OFF_BBC, OFF_RANGES = 2048, 2624, 2816, 4096

    def __init__(self, rank: int, world: int, n: int, device, theta: torch.Tensor, stage_ptrs: Sequence[int],
                 stage_mc: int, ctl: torch.Tensor, ctl_ptrs: Sequence[int], stream: Optional[torch.cuda.Stream] = None,
                 fused: Optional[bool] = None):
        from ..ops import _lib
        from ..ops._lib import c_int, c_void, c_ll
        self.L = _lib.lib()
        u64 = ctypes.c_ulonglong
        _lib.register("dt_dm_range", [c_void, c_int, c_ll, c_ll, c_void, c_void])
        _lib.register("dt_dm_wait", [c_void, u64, c_int, u64, c_void])
        _lib.register("dt_dm_apply", [c_void, c_int, c_ll, c_void, c_ll, c_ll, c_void, c_void, c_int, c_int, c_void])
        _lib.register("dt_dm_broadcast", [c_void, c_ll, c_ll, c_void, c_void, c_int, c_void, c_void, c_void])
        _lib.register("dt_dm_fused", [c_void, c_int, c_void, c_void, c_ll, c_ll, c_void, c_void, c_void, c_void, c_int,
                                      c_void, c_void, c_void])
        _lib.register("dt_dm_tile_elems", [], ctypes.c_longlong)
        assert world <= 8 and ctl.numel() >= self.CTL_BYTES
        self.rank, self.world, self.n = rank, world, n
        self.device = torch.device(device)
        self.theta = theta
        self.stage_ptrs, self.stage_mc = list(stage_ptrs), int(stage_mc or 0)
        self.ctl, self.ctl_ptrs = ctl, list(ctl_ptrs)
        self.base = ctl.data_ptr()
        self.a, self.b = self.range_of(rank)
        self.stream = stream or torch.cuda.Stream(device=self.device, priority=-100)
        self.coef_host = torch.zeros(64, dtype=torch.float32).pin_memory()
        self.coef_dev = ctl[self.OFF_COEF:self.OFF_COEF + 256].view(torch.float32)
        self._keep = None
        # fused tile path (dt_dm_fused): one pass over the slice that sums every member in shared memory and
        # writes each tile once, locally and to every node; DT_DM_FUSED=1 selects it by default
        self.fused = (os.environ.get("DT_DM_FUSED", "0") == "1") if fused is None else bool(fused)
        self.tile = int(self.L.dt_dm_tile_elems())
        self.bounds = torch.empty(0, dtype=torch.int64, device=self.device)

    def range_of(self, r: int):
        n4 = self.n // 4
        return (r * n4 // self.world) * 4, ((r + 1) * n4 // self.world) * 4

    def _pack(self, contribs: List[Contribution]):
        raw = b"".join(struct.pack(_CONTRIB_FMT, c.idx_ptr if not c.dense else 0, c.q_ptr, c.val_ptr, c.scales_ptr,
                                   c.win_ptr if not c.dense else 0, c.count, max(c.block, 1), int(c.dense), 1.0, 0)
                       for c in contribs)
        buf = ctypes.create_string_buffer(raw, len(raw))
        self._keep = buf
        return buf

    def apply(self, contribs: List[Contribution], coefs: Sequence[float], outer_lr: float):
        """This node's slice: theta[a, b) -= outer_lr * sum_c coef_c * x_c, then its broadcast into every node's
        slot; enqueued on ``self.stream``."""
        from ..ops._lib import check
        n = len(contribs)
        assert 0 < n <= 64 and len(coefs) == n
        buf = self._pack(contribs)
        sp = self.stream.cuda_stream
        has_dense = any(c.dense for c in contribs)
        has_sparse = any(not c.dense for c in contribs)
        max_len = max(max((self.b - self.a) if c.dense else c.count // self.world + 1 for c in contribs), 1)
        self.stream.synchronize()  # the pinned coefficient staging buffer is reused
        self.coef_host[:n] = torch.tensor([-float(outer_lr) * k for k in coefs], dtype=torch.float32)
        with torch.cuda.stream(self.stream):
            self.coef_dev[:n].copy_(self.coef_host[:n], non_blocking=True)
            ranges = self.base + self.OFF_RANGES
            if has_sparse:
                check(self.L.dt_dm_range(buf, n, self.a, self.b, ranges, sp), "dt_dm_range")
            dests = (ctypes.c_void_p * self.world)(*self.stage_ptrs)
            if self.fused:
                need = n * ((self.b - self.a + self.tile - 1) // self.tile + 1)
                if self.bounds.numel() < need:
                    self.bounds = torch.empty(need, dtype=torch.int64, device=self.device)
                check(self.L.dt_dm_fused(buf, n, ranges, self.bounds.data_ptr(), self.a, self.b,
                                         self.coef_dev.data_ptr(), self.theta.data_ptr(), self.stage_mc or None, dests,
                                         self.world, self.ctl_ptrs[0] + self.OFF_DONE, self.base + self.OFF_BBC, sp),
                      "dt_dm_fused")
                return
            check(self.L.dt_dm_apply(buf, n, max_len, ranges, self.a, self.b, self.coef_dev.data_ptr(),
                                     self.theta.data_ptr(), int(has_dense), int(has_sparse), sp), "dt_dm_apply")
            check(self.L.dt_dm_broadcast(self.theta.data_ptr(), self.a, self.b, self.stage_mc or None, dests,
                                         self.world, self.ctl_ptrs[0] + self.OFF_DONE, self.base + self.OFF_BBC, sp),
                  "dt_dm_broadcast")

    def check(self, what: str = "apply"):
        """Synchronise this node's merge stream; raise on a recorded device error."""
        from .. import ops
        self.stream.synchronize()
        err = ops.device_error(self.stream)
        if err[0]:
            raise RuntimeError(f"distributed merge ({what}): device error {err}")

    def finish(self, att: int):
        """Rank 0, after every node's ``apply`` of attempt ``att`` (the att-th on this merger) completed."""
        from ..ops._lib import check
        with torch.cuda.stream(self.stream):
            check(self.L.dt_dm_wait(self.base + self.OFF_DONE, att * self.world, 912, DT_WAIT_SHORT_NS,
                                    self.stream.cuda_stream), "dt_dm_wait")
        self.check("finish")

    def run_local(self, contribs: List[Contribution], stats: List[List[float]], outer_lr: float, att: int):
        """The whole attempt on a single node (world 1): plan from ``stats``, apply, finish."""
        assert self.world == 1
        coefs, info = DeviceMerger.plan(contribs, stats)
        self.apply(contribs, coefs, outer_lr)
        self.finish(att)
        info["pulled_bytes"] = sum(c.wire_bytes for c in contribs)
        return info
