"""Node runtime over the coordinator HTTP API + object store (reference node/cli/src/continuous.rs).

Three concurrent activities, as in the reference (continuous.rs:74-344, 379-675):
* checkpoint manager - polls GET /checkpoint/latest every ``poll_secs``, downloads new checkpoints;
* uploader           - compresses each finished round (EF -> top-k -> INT8), uploads it to the store
                       (or through the coordinator's /upload proxy), then POST /delta; measures upload
                       bandwidth for the bandwidth-adaptive policy (raw if it fits a 10 s budget, else
                       adaptive_top_k, trainer.rs:33-70) and recommends H_mini for ~10 s uploads;
* training loop      - continuous steps; every ``h_mini`` steps it snapshots the round delta and hands it
                       to the uploader without waiting; on a new checkpoint it pushes the partial round,
                       swaps weights and restarts AdamW and error feedback; heartbeat every 10 steps.

Backends: ``cpu`` (fp32 oracle model + reference AdamW, the micro-test configuration) and ``cuda``
(the sm_100a ``TrainEngine``).
"""
from __future__ import annotations

import math
import os
import queue
import threading
import time
from typing import Callable, Dict, List, Optional

import torch

from .. import protocol as P
from ..config import CompressionConfig, ModelConfig, OptimConfig
from ..coordinator.client import CoordinatorClient
from ..models.params import ParamLayout
from ..utils.checkpoint import load_safetensors_bytes
from ..utils.delta_codec import encode_sparse_delta
from .compression import adaptive_top_k, compress_reference  # noqa: F401 (adaptive_top_k re-exported)
from ..utils.resources import memory_pressure
from ..utils.watchdog import StepWatchdog, watchdog_limit


class CpuBackend:
    """fp32 oracle model + reference-semantics AdamW on the host."""

    def __init__(self, cfg: ModelConfig, optim: OptimConfig):
        from ..models import oracle
        self.oracle, self.cfg, self.optim = oracle, cfg, optim
        self.layout = ParamLayout(cfg)
        self.params: Dict[str, torch.Tensor] = {}
        self.opt = None

    def load(self, sd: Dict[str, torch.Tensor]):
        self.params = {k: v.detach().clone().float().requires_grad_() for k, v in sd.items()}
        o = self.optim
        self.opt = self.oracle.AdamWRef(self.params, lr=o.lr, betas=(o.beta1, o.beta2), eps=o.eps,
                                        weight_decay=o.weight_decay, clip=o.grad_clip_norm, clip_global=o.clip_global)

    def state(self) -> Dict[str, torch.Tensor]:
        return {k: v.detach().clone() for k, v in self.params.items()}

    def loss(self, tokens: torch.Tensor) -> float:
        with torch.no_grad():
            return float(self.oracle.lm_loss(self.params, self.cfg, tokens.long()).item())

    def optimizer_state(self):
        return {"m": {k: t.clone() for k, t in self.opt.m.items()}, "v": {k: t.clone() for k, t in self.opt.v.items()},
                "t": self.opt.t}

    def load_optimizer_state(self, st):
        for k in self.opt.m:
            self.opt.m[k].copy_(st["m"][k])
            self.opt.v[k].copy_(st["v"][k])
        self.opt.t = int(st["t"])

    def step(self, tokens: torch.Tensor, lr: float, max_loss: Optional[float] = None) -> float:
        """One step; a non-finite loss, or one above ``max_loss`` (a spike), returns without an update."""
        loss = self.oracle.lm_loss(self.params, self.cfg, tokens.long())
        if not math.isfinite(loss.item()):
            for p in self.params.values():
                p.grad = None
            return float("nan")
        if max_loss is not None and loss.item() > max_loss:
            return float(loss.item())
        loss.backward()
        self.opt.step(lr)
        return float(loss.item())


class CudaBackend:
    """The sm_100a training engine (fp32 master, bf16 compute)."""

    def __init__(self, cfg: ModelConfig, optim: OptimConfig, batch: int, seq_len: int, device):
        from ..models.engine import TrainEngine
        self.eng = TrainEngine(cfg, batch, seq_len, optim=optim, device=device)
        self.layout = self.eng.layout
        self.cfg = cfg

    def load(self, sd):
        flat = torch.zeros(self.layout.total)
        self.layout.load_state_dict(flat, sd)
        self.eng.load_flat(flat)

    def state(self):
        return self.layout.to_state_dict(self.eng.master)

    def optimizer_state(self):
        """AdamW moments and the device hyper-parameter block (step count, bias corrections)."""
        return {"m": self.eng.m.detach().cpu().clone(), "v": self.eng.v.detach().cpu().clone(),
                "hp": self.eng.hp.detach().cpu().clone()}

    def load_optimizer_state(self, st):
        with torch.no_grad():
            self.eng.m.copy_(st["m"].to(self.eng.device))
            self.eng.v.copy_(st["v"].to(self.eng.device))
            self.eng.hp.copy_(st["hp"].to(self.eng.device))

    def step(self, tokens, lr, max_loss=None):
        # the fused step updates before the loss is read: a spike is only excluded from the round's
        # statistics here, while a non-finite loss skips the update on the device
        self.eng.set_lr(lr)
        self.eng.set_tokens(tokens.to(self.eng.device, non_blocking=True))
        self.eng.step()
        return float(self.eng.loss[0].item())

    # ── round deltas compressed on the device (reference continuous.rs:190-219 semantics) ──
    # The round-start snapshot and the error-feedback residual live on the GPU (DeviceCompressor); a push
    # forms delta + EF, selects the exact per-tensor top-k and compacts it there, and only the kept
    # (index, value) pairs cross to the host (8 bytes per kept entry), where the reference's per-tensor
    # INT8 step and the JSON/zstd encoding run on k values instead of the whole model.
    def enable_device_compression(self, cfg: CompressionConfig, max_fraction: float = 1.0):
        from .compression import DeviceCompressor, DevicePayload
        self.dcfg = CompressionConfig(top_k_fraction=cfg.top_k_fraction, quantize_int8=False,
                                      per_tensor_adaptive=cfg.per_tensor_adaptive, int8_block=0,
                                      zstd_level=cfg.zstd_level)
        cap = DeviceCompressor.capacity_for(self.layout, max_fraction)
        self.dcomp = DeviceCompressor(self.layout, self.eng.device, self.dcfg,
                                      payload=DevicePayload.allocate(cap, 0, self.eng.device))
        self.dcomp.reset(self.eng.master)
        self.cstream = torch.cuda.Stream(device=self.eng.device)
        self._payload_free = None      # event: the host has copied the previous payload out
        self._host_idx = self._host_val = None
        self.d2h_bytes_last = 0
        offs = [(e.offset, e.numel, e.name, list(e.shape)) for e in self.layout.entries]
        self._entries = sorted(offs)
        self._starts = torch.tensor([o for o, _, _, _ in self._entries], dtype=torch.int64)

    def round_reset(self, clear_ef: bool = False):
        """New round start at the current weights (snapshot <- master); ``clear_ef`` also restarts the error
        feedback (a checkpoint boundary)."""
        if clear_ef:
            self.dcomp.reset(self.eng.master)
        else:
            self.dcomp.snap.copy_(self.eng.master)

    def compress_round(self, k_fraction: float):
        """Delta (snapshot - master) + error feedback -> exact top-k on the device; returns a handle the
        uploader thread passes to ``collect``. The snapshot becomes the current weights."""
        train = torch.cuda.current_stream(self.eng.device)
        if self._payload_free is not None:
            self.cstream.wait_event(self._payload_free)   # the previous payload has been read out
        self.dcomp.begin(self.eng.master, stream=train)     # pass A: ordered with the training steps
        ev = torch.cuda.Event()
        ev.record(train)
        self.cstream.wait_event(ev)
        self.dcomp.finish(stream=self.cstream, k_fraction=k_fraction, quant_block=0)
        done = torch.cuda.Event()
        done.record(self.cstream)
        return done, k_fraction

    def collect(self, handle, cfg: CompressionConfig, want_ef: bool = False):
        """(SparseDeltaT, stats[, EF state dict]) of a ``compress_round`` handle, on the calling thread."""
        from .compression import SparseDeltaT, quantize_int8, dequantize_int8
        done, kf = handle
        done.synchronize()
        st = self.dcomp.read_stats(raw=False, quantized=False)
        k = int(st["num_params_kept"])
        if self._host_idx is None or self._host_idx.numel() < k:
            n = max(k, 1)
            self._host_idx = torch.empty(n, dtype=torch.int32).pin_memory()
            self._host_val = torch.empty(n, dtype=torch.float32).pin_memory()
        p = self.dcomp.payload
        with torch.cuda.stream(self.cstream):
            self._host_idx[:k].copy_(p.idx[:k], non_blocking=True)
            self._host_val[:k].copy_(p.val[:k], non_blocking=True)
            ef = None
            if want_ef:
                ef = {e.name: self.dcomp.ef[e.offset:e.offset + e.numel].view(e.shape).float().cpu()
                      for e in self.layout.entries}
            freed = torch.cuda.Event()
            freed.record(self.cstream)
        freed.synchronize()
        self._payload_free = freed
        self.d2h_bytes_last = 8 * k
        flat = self._host_idx[:k].to(torch.int64)
        vals = self._host_val[:k].clone()
        pos = torch.searchsorted(self._starts, flat, right=True) - 1
        bounds = torch.searchsorted(pos, torch.arange(len(self._entries) + 1), right=False)
        idxs, values, shapes, scales = {}, {}, {}, ({} if cfg.quantize_int8 else None)
        for j, (off, numel, name, shape) in enumerate(self._entries):
            a, b = int(bounds[j]), int(bounds[j + 1])
            shapes[name] = shape
            idxs[name] = flat[a:b] - off
            v = vals[a:b]
            if cfg.quantize_int8:   # the reference's per-tensor scale, values shipped dequantised
                q, s = quantize_int8(v, 0)
                v = dequantize_int8(q, s, 0)
                scales[name] = float(s[0])
            values[name] = v
        sd = SparseDeltaT(indices=idxs, values=values, shapes=shapes, scales=scales,
                          config=CompressionConfig(top_k_fraction=kf, quantize_int8=cfg.quantize_int8,
                                                   per_tensor_adaptive=cfg.per_tensor_adaptive,
                                                   zstd_level=cfg.zstd_level))
        stats = {"dense_norm": st["dense_norm"], "sparse_norm": st["sparse_norm"],
                 "retention_ratio": st["retention_ratio"], "top_k_fraction": kf,
                 "num_params_total": st["num_params_total"], "num_params_kept": k,
                 "raw_param_bytes": 4 * st["num_params_total"]}
        return (sd, stats, ef) if want_ef else (sd, stats)

    def load_ef(self, ef):
        for e in self.layout.entries:
            self.dcomp.ef[e.offset:e.offset + e.numel].copy_(ef[e.name].reshape(-1).to(self.eng.device))


class HttpNode:
    def __init__(self, coordinator_url: str, store, model_cfg: ModelConfig, batch: int, seq_len: int,
                 h_mini: int = 50, optim: Optional[OptimConfig] = None, compression: Optional[CompressionConfig] = None,
                 device: str = "cpu", node_id: Optional[str] = None, data: Optional[Callable[[], torch.Tensor]] = None,
                 poll_secs: float = 5.0, use_upload_proxy: bool = False, bandwidth_adaptive: bool = False,
                 heartbeat_every: int = 10, loss_based_lr: Optional[bool] = None,
                 expected_step_secs: Optional[float] = None, resume_path: Optional[str] = None,
                 resume_every: int = 1, max_memory_fraction: float = 0.80,
                 h_mini_bounds: Optional[tuple] = None, ckpt_cache_dir: Optional[str] = None):
        self.client = CoordinatorClient(coordinator_url)
        self.store = store
        self.cfg, self.batch, self.seq_len, self.h_mini = model_cfg, batch, seq_len, h_mini
        self.optim = optim or OptimConfig()
        self.comp = compression or CompressionConfig(top_k_fraction=0.1)
        self.dev = device
        self.backend = CpuBackend(model_cfg, self.optim) if device == "cpu" else \
            CudaBackend(model_cfg, self.optim, batch, seq_len, device)
        # a GPU node compresses its round deltas on the device: only the kept entries leave the GPU
        self.device_comp = isinstance(self.backend, CudaBackend)
        if self.device_comp:
            self.backend.enable_device_compression(self.comp, 1.0 if bandwidth_adaptive else
                                                   max(self.comp.top_k_fraction, 0.0))
        self.data = data
        self.poll_secs, self.use_proxy, self.bw_adaptive = poll_secs, use_upload_proxy, bandwidth_adaptive
        self.hb_every = heartbeat_every
        # inner lr mode: constant (default) or loss-based (LR_MODE=loss_based, reference continuous.rs:586-596)
        self.loss_based_lr = (os.environ.get("LR_MODE") == "loss_based") if loss_based_lr is None else loss_based_lr
        self.expected_step_secs = expected_step_secs
        self.node_id = node_id
        self.version = -1
        self.seq = 0
        self.global_step = 0
        self.stop = threading.Event()
        self.new_ckpt: "queue.Queue" = queue.Queue()
        self.up_q: "queue.Queue" = queue.Queue()
        self.bandwidth_bps = 0.0
        self.recommended_h_mini = h_mini
        self.log: List[dict] = []
        self.pushes: List[dict] = []
        self.errors: List[str] = []
        self._ef: Dict[str, torch.Tensor] = {}
        self._ef_gen = 0        # bumped by the training loop at each checkpoint swap
        self._ef_gen_seen = 0   # generation the uploader's error buffer belongs to
        self._threads: List[threading.Thread] = []
        # node-local resume file: written by the uploader after every `resume_every`-th full-round push
        self.resume_path, self.resume_every = resume_path, max(int(resume_every), 1)
        self.max_memory_fraction = max_memory_fraction  # host memory: stop above this + 10 % used
        # (min, max) inner steps: at each checkpoint swap the push interval follows the bandwidth-based
        # recommendation (steps whose delta uploads in ~10 s), clamped to these bounds (continuous.rs:936-945)
        self.h_mini_bounds = h_mini_bounds
        self.spikes_skipped = 0
        # checkpoints fetched from the store are kept here, the newest 3 (continuous.rs:966-995)
        self.ckpt_cache_dir = ckpt_cache_dir
        self.resumed: Optional[str] = None   # "exact" (same checkpoint: weights, AdamW, EF restored) / "identity"
        self._resume_rec = self._read_resume()
        if self.node_id is None and self._resume_rec is not None:
            self.node_id = self._resume_rec["node_id"]  # register under the same identity

    # ─────────── lifecycle ───────────
    def register(self, gpu_model: str = "cpu", vram_gb: float = 0.0):
        req = P.RegisterRequest(gpu_model=gpu_model, gpu_memory_gb=vram_gb, bandwidth_mbps=0.0, node_id=self.node_id,
                                hardware={"gpu_model": gpu_model, "vram_mb": int(vram_gb * 1024),
                                          "device_type": "Cpu" if self.dev == "cpu" else "DiscreteGpu",
                                          "cpu_cores": 1, "ram_mb": 0, "h_mini": self.h_mini,
                                          "batch_size": self.batch})
        r = self.client.register(req)
        self.node_id = r.node_id
        return r

    def _load_version(self, v: int):
        if not self.ckpt_cache_dir:
            return load_safetensors_bytes(self.store.get(P.checkpoint_path(v)))
        d = os.path.join(self.ckpt_cache_dir, "checkpoints")
        path = os.path.join(d, f"v{v}.safetensors")
        if os.path.exists(path):
            with open(path, "rb") as f:
                return load_safetensors_bytes(f.read())
        data = self.store.get(P.checkpoint_path(v))
        os.makedirs(d, exist_ok=True)
        with open(path + ".tmp", "wb") as f:
            f.write(data)
        os.replace(path + ".tmp", path)
        cached = sorted((int(n[1:-len(".safetensors")]) for n in os.listdir(d)
                         if n.startswith("v") and n.endswith(".safetensors")), reverse=True)
        for old in cached[3:]:
            try:
                os.remove(os.path.join(d, f"v{old}.safetensors"))
            except OSError:
                pass
        return load_safetensors_bytes(data)

    def _ckpt_manager(self):
        while not self.stop.wait(self.poll_secs):
            try:
                info = self.client.get_latest_checkpoint()
                if info.version > self.version:
                    self.new_ckpt.put((info.version, self._load_version(info.version)))
            except Exception as e:
                self.errors.append(f"ckpt: {e}")

    def _uploader(self):
        while not self.stop.is_set() or not self.up_q.empty():
            try:
                pkg = self.up_q.get(timeout=0.05)
            except queue.Empty:
                continue
            try:
                self._compress_upload_push(pkg)
            except Exception as e:
                self.errors.append(f"upload: {e}")

    def _push_fraction(self, mean_loss: float):
        """(top-k fraction, quantise) of the next device-compressed push: the configured top-k, or with
        the bandwidth-adaptive policy the decision of ``adaptive_push_mode`` from the measured upload
        bandwidth and the raw delta size (4 bytes per parameter; no trial compression)."""
        from .compression import adaptive_push_mode
        n = self.backend.layout.num_params()
        kind, kf, qb = adaptive_push_mode(self.bw_adaptive, self.bandwidth_bps, 4 * n, mean_loss, self.comp)
        if kind == "raw":
            return 1.0, False
        return kf, (self.comp.quantize_int8 and (not self.bw_adaptive or self.bandwidth_bps <= 0))

    def _compress_upload_push(self, pkg):
        delta, shapes, push, mean_loss, ef_generation, snap = pkg
        if isinstance(delta, tuple) and delta and delta[0] == "device":
            _, handle, quant = delta
            cfg = CompressionConfig(top_k_fraction=handle[1], quantize_int8=quant,
                                    per_tensor_adaptive=self.comp.per_tensor_adaptive, zstd_level=self.comp.zstd_level)
            if snap is not None:
                sd, stats, ef = self.backend.collect(handle, cfg, want_ef=True)
                self._ef = ef
            else:
                sd, stats = self.backend.collect(handle, cfg)
            self._upload_and_push(sd, cfg, stats, push, snap)
            return
        if ef_generation != self._ef_gen_seen:   # error feedback restarts at a checkpoint boundary
            self._ef, self._ef_gen_seen = {}, ef_generation
        cfg = self.comp
        raw_bytes = sum(t.numel() for t in delta.values()) * 4
        if self.bw_adaptive and self.bandwidth_bps > 0:
            budget = int(self.bandwidth_bps * 10)
            trial_cfg = CompressionConfig(top_k_fraction=1.0, quantize_int8=False, zstd_level=cfg.zstd_level)
            trial, _ = compress_reference(delta, shapes, trial_cfg, dict(self._ef))
            if len(encode_sparse_delta(trial, trial_cfg.zstd_level)) <= budget:
                cfg = trial_cfg
            else:
                cfg = CompressionConfig(top_k_fraction=adaptive_top_k(mean_loss, budget, raw_bytes),
                                        quantize_int8=False, zstd_level=cfg.zstd_level)
        sd, stats = compress_reference(delta, shapes, cfg, self._ef)
        self._upload_and_push(sd, cfg, stats, push, snap)

    def _upload_and_push(self, sd, cfg, stats, push, snap):
        blob = encode_sparse_delta(sd, cfg.zstd_level)
        t0 = time.time()
        for attempt in range(5):   # 5 retries with backoff (continuous.rs:244-283)
            try:
                if self.use_proxy:
                    self.client.upload(push.delta_key, blob)
                else:
                    self.store.put(push.delta_key, blob)
                break
            except Exception:
                if attempt == 4:
                    raise
                time.sleep(2 ** attempt * 0.1)
        secs = max(time.time() - t0, 1e-6)
        self.bandwidth_bps = len(blob) / secs
        self.recommended_h_mini = int(min(max(10.0 / secs * push.inner_steps, 10), 500))
        push.compressed_bytes, push.dense_norm, push.sparse_norm = len(blob), stats["dense_norm"], stats["sparse_norm"]
        resp, accepted = None, False
        for attempt in range(5):   # push retries with backoff (continuous.rs:284-311)
            try:
                resp = self.client.push_delta(push)
                accepted = resp.accepted
                # a retry whose earlier attempt landed (reply lost) meets the coordinator's dedup by sequence
                # number: that push was delivered
                if not accepted and attempt > 0 and (resp.reason or "").startswith(
                        f"Duplicate: existing seq_num {push.seq_num} >="):
                    accepted = True
                break
            except Exception:
                if attempt == 4:
                    raise
                time.sleep(2 ** attempt * 0.1)
        self.pushes.append({"seq": push.seq_num, "version": push.checkpoint_version, "accepted": accepted,
                            "reason": resp.reason, "bytes": len(blob), "retention": stats["retention_ratio"],
                            "top_k": cfg.top_k_fraction})
        if snap is not None:
            self._write_resume(snap, push.seq_num)

    # ─────────── node-local resume ───────────
    def _write_resume(self, snap, seq: int):
        """Weights and AdamW state at a round boundary, the error-feedback residual after that round's push,
        the data position and the node's identity, written atomically."""
        rec = dict(snap, format=1, node_id=self.node_id, seq=seq,
                   ef={k: v.clone() for k, v in self._ef.items()})
        tmp = self.resume_path + ".tmp"
        torch.save(rec, tmp)
        os.replace(tmp, self.resume_path)

    def _read_resume(self):
        if not self.resume_path or not os.path.exists(self.resume_path):
            return None
        try:
            rec = torch.load(self.resume_path, weights_only=False)
        except Exception as e:
            self.errors.append(f"resume file unreadable: {e}")
            return None
        shapes = {e.name: tuple(e.shape) for e in ParamLayout(self.cfg).entries}
        if rec.get("format") != 1 or {k: tuple(v.shape) for k, v in rec["weights"].items()} != shapes:
            self.errors.append("resume file is for another model; ignored")
            return None
        return rec

    def _apply_resume(self, rec, latest_version: int):
        """Same checkpoint as when the file was written: continue exactly (weights, AdamW, EF). Newer
        checkpoint: load it as a swap would (fresh AdamW, EF restarts) and keep identity and data position."""
        self.seq = int(rec["seq"])
        self.global_step = int(rec["global_step"])
        src = getattr(self.data, "__self__", None)
        if rec.get("data") is not None and src is not None and hasattr(src, "restore"):
            src.restore(rec["data"])
        if int(rec["version"]) == latest_version:
            self.backend.load(rec["weights"])
            self.backend.load_optimizer_state(rec["optimizer"])
            self._ef = {k: v.clone() for k, v in rec["ef"].items()}
            if self.device_comp:
                self.backend.round_reset()
                self.backend.load_ef(self._ef)
            self.resumed = "exact"
            return True
        self.resumed = "identity"
        return False

    # ─────────── training loop ───────────
    def _round_start(self, boundary: bool = False):
        """Round-start weights: a host copy (CPU backend) or, compressing on the device, the device
        snapshot (``boundary``: a new checkpoint, the error feedback restarts too)."""
        if self.device_comp:
            self.backend.round_reset(clear_ef=boundary)
            return None
        return self.backend.state()

    def _build_push(self, start, steps, tokens, losses, t0, boundary: bool = False):
        mean_loss = sum(losses) / len(losses) if losses else 0.0
        want_snap = boundary and self.resume_path and (self.seq + 1) % self.resume_every == 0
        if self.device_comp:
            kf, quant = self._push_fraction(mean_loss)
            delta, shapes = ("device", self.backend.compress_round(kf), quant), None
            cur = self.backend.state() if want_snap else None
        else:
            cur = self.backend.state()
            delta = {k: (start[k].reshape(-1) - cur[k].reshape(-1)).float() for k in start}
            shapes = {k: list(v.shape) for k, v in start.items()}
        self.seq += 1
        snap = None
        if want_snap:
            src = getattr(self.data, "__self__", None)
            snap = {"weights": {k: v.detach().float().cpu().clone() for k, v in cur.items()},
                    "optimizer": self.backend.optimizer_state(), "global_step": self.global_step,
                    "version": self.version,
                    "data": src.state() if src is not None and hasattr(src, "state") else None}
        push = P.DeltaPush(node_id=self.node_id, seq_num=self.seq, checkpoint_version=self.version,
                           inner_steps=steps, delta_key=P.delta_path(self.version, self.node_id, self.seq),
                           training_loss=mean_loss, tokens_processed=tokens, training_time_secs=time.time() - t0)
        self.up_q.put((delta, shapes, push, mean_loss, self._ef_gen, snap))

    def run(self, total_steps: int, stop_on_version: Optional[int] = None):
        """Train ``total_steps`` steps continuously (or until ``stop_on_version`` is reached)."""
        rec = self._resume_rec if self.version < 0 else None
        self._resume_rec = None
        if self.node_id is None:
            self.register()
        exact = False
        if self.version < 0:
            info = self.client.get_latest_checkpoint()
            self.version = info.version
            exact = rec is not None and self._apply_resume(rec, info.version)
            if not exact:
                self.backend.load(self._load_version(info.version))
        for fn in (self._ckpt_manager, self._uploader):
            t = threading.Thread(target=fn, daemon=True)
            t.start()
            self._threads.append(t)
        warm = max(int(self.h_mini * self.optim.warmup_fraction), 2)
        first_round = rec is None  # a resumed node has had its warm-up
        start, round_step, round_tokens, losses, t0 = self._round_start(boundary=not exact), 0, 0, [], time.time()
        loss_ema, loss_count = 0.0, 0
        ln_vocab = math.log(self.cfg.vocab_size)
        wd = None
        if self.expected_step_secs is not None:  # per-step watchdog (reference trainer.rs:1098-1163)
            wd = StepWatchdog(watchdog_limit(self.expected_step_secs), on_timeout=self._hung)
        try:
            while self.global_step < total_steps:
                if wd is not None:
                    wd.beat()
                if self.stop.is_set():
                    break
                try:
                    v, sd = self.new_ckpt.get_nowait()
                except queue.Empty:
                    v = None
                if v is not None and v > self.version:
                    if round_step > 0 and losses:
                        self._build_push(start, round_step, round_tokens, losses, t0)
                    self.backend.load(sd)          # fresh AdamW, like the reference's re-entered loop
                    self._ef_gen += 1
                    self.version = v
                    if self.h_mini_bounds is not None:
                        lo, hi = self.h_mini_bounds
                        self.h_mini = int(min(max(self.recommended_h_mini, lo), hi))
                    start, round_step, round_tokens, losses, t0 = self._round_start(boundary=True), 0, 0, [], time.time()
                    if stop_on_version is not None and v >= stop_on_version:
                        break
                if round_step >= self.h_mini:
                    if not (first_round and round_step <= warm):
                        self._build_push(start, round_step, round_tokens, losses, t0, boundary=True)
                    if first_round and round_step <= warm and self.device_comp:
                        self.backend.round_reset()  # the skipped warm-up round's steps are not pushed
                    start = None if self.device_comp else self.backend.state()
                    round_step, round_tokens, losses, t0 = 0, 0, [], time.time()
                    first_round = False
                tokens = self.data()
                if first_round and round_step < warm:
                    lr = self.optim.lr * round_step / warm
                elif self.loss_based_lr and loss_ema > 0.0:
                    lr = self.optim.lr * min(max(loss_ema / ln_vocab, 0.1), 1.0)
                else:
                    lr = self.optim.lr
                # a loss above both 3x and +5 of its EMA is a spike: no update (continuous.rs:607-621)
                spike_at = max(loss_ema * 3.0, loss_ema + 5.0) if loss_count > 3 else None
                loss = self.backend.step(tokens, lr, spike_at)
                if not math.isfinite(loss):
                    continue  # NaN loss: the update was skipped
                if spike_at is not None and loss > spike_at:
                    self.spikes_skipped += 1
                    continue
                losses.append(loss)
                loss_count += 1
                loss_ema = loss if loss_count == 1 else loss_ema * 0.9 + loss * 0.1
                round_step += 1
                self.global_step += 1
                round_tokens += self.batch * self.seq_len
                self.log.append({"step": self.global_step, "loss": loss, "version": self.version, "lr": lr})
                if self.global_step % self.hb_every == 0:
                    threading.Thread(target=self._heartbeat, args=(round_step, loss), daemon=True).start()
                    if memory_pressure(self.max_memory_fraction):  # reference main.rs:723-734
                        self.errors.append(f"host memory pressure: above {self.max_memory_fraction + 0.1:.0%} used; "
                                           "stopping")
                        break
        finally:
            if wd is not None:
                wd.close()
            self.stop.set()
            for t in self._threads:
                t.join(timeout=120)
        return self.log

    def _hung(self, stalled: float):
        self.errors.append(f"GpuHung: no step for {stalled:.0f} s")
        self.stop.set()

    def _heartbeat(self, step, loss):
        try:
            self.client.heartbeat_sync(P.HeartbeatRequest(node_id=self.node_id, step=step, total_steps=self.h_mini,
                                                          loss=loss, checkpoint_version=self.version))
        except Exception:
            pass  # heartbeat failures are non-fatal (continuous.rs:650-673)
