"""Coordinator service: the reference's 10-route HTTP API over the native HTTP server core.

Routes, bodies and status codes follow coordinator/src/routes.rs:22-537; state handling follows
state.rs; aggregation follows aggregation.rs:154-472 (download checkpoint + deltas, decode, validate,
3x running-average clip, staleness x tokens weighted average, Nesterov apply with lr 1 / momentum 0,
upload checkpoint + velocity + metadata, JSONL stats, background housekeeping); persistence follows
main.rs:42-139 (load at start, 30 s background flush, flush before and after each aggregation).

Deliberate difference: pushes that arrive while an aggregation runs are applied to the next cycle
(``Accumulator`` carry-over) instead of being wiped by the post-aggregation reset.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import logging
import math
import threading
import time
import traceback
import uuid
from typing import Dict, Optional, Tuple

import torch

from ..config import CoordinatorConfig, TrainingParams
from .. import protocol as P
from ..utils import native
from ..utils.storage import ObjectStore, StorageError
from ..utils.checkpoint import load_safetensors_bytes, save_safetensors, save_velocity, load_velocity
from ..utils.delta_codec import decode_delta, decode_dtz_dense, LowRankPayload
from ..parallel.merge import merge_reference
from .metrics import Metrics

VERSION = "0.1.0"

_HANDLER = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_void_p,
                            ctypes.c_longlong, ctypes.c_void_p)


log = logging.getLogger("distrain_b200.coordinator")

class CoordinatorService:
    def __init__(self, cfg: CoordinatorConfig, store: ObjectStore, merge_device: str = "cpu",
                 flush_interval: float = 30.0):
        self.cfg, self.store = cfg, store
        self.merge_device = merge_device
        self.metrics = Metrics()
        self.lock = threading.RLock()
        self.acc = P.Accumulator(staleness_decay=cfg.staleness_decay, max_staleness=cfg.max_staleness,
                                 min_contributions=cfg.min_contributions)
        self._load_state()
        self.agg_thread: Optional[threading.Thread] = None
        self.server = None
        self._cb = None
        self.flush_interval = flush_interval
        self._stop = threading.Event()
        self._flusher = None
        self.last_error: Optional[str] = None

    # ─────────── persistence ───────────
    def _load_state(self):
        try:
            self.acc.state = P.AccumulatorState.from_dict(self.store.get_json(P.accumulator_path()))
        except (StorageError, ValueError, KeyError):
            self.acc.state = P.AccumulatorState()
        try:
            self.acc.cs = P.CoordinatorPersistentState.from_dict(self.store.get_json(P.coordinator_state_path()))
        except (StorageError, ValueError, KeyError):
            self.acc.cs = P.CoordinatorPersistentState()
        self.metrics.checkpoint_version = self.acc.state.checkpoint_version

    def flush(self):
        with self.lock:
            a = self.acc.state.to_dict()
            c = self.acc.cs.to_dict()
        try:
            self.store.put_json(P.accumulator_path(), a)
            self.store.put_json(P.coordinator_state_path(), c)
        except Exception as e:  # best effort, like the reference's background flush
            self.last_error = f"flush: {e}"

    def _flush_loop(self):
        while not self._stop.wait(self.flush_interval):
            self.flush()

    # ─────────── HTTP plumbing ───────────
    def start(self, host: Optional[str] = None, port: Optional[int] = None, threads: int = 8) -> int:
        L = native.rt()
        native.register("dtr_http_start", [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, _HANDLER,
                                           ctypes.c_void_p], ctypes.c_void_p)
        native.register("dtr_http_port", [ctypes.c_void_p], ctypes.c_int)
        native.register("dtr_http_stop", [ctypes.c_void_p], None)
        native.register("dtr_http_respond", [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_void_p,
                                             ctypes.c_longlong], None)
        self._cb = _HANDLER(self._on_request)
        h = L.dtr_http_start((host or self.cfg.host).encode(), self.cfg.port if port is None else port, threads,
                             512 << 20, self._cb, None)
        if not h:
            raise RuntimeError("coordinator: cannot bind HTTP port")
        self.server = h
        self.port = L.dtr_http_port(h)
        self._flusher = threading.Thread(target=self._flush_loop, daemon=True)
        self._flusher.start()
        return self.port

    def stop(self):
        self._stop.set()
        if self.agg_thread is not None:
            self.agg_thread.join(timeout=60)
        if self.server:
            native.rt().dtr_http_stop(self.server)
            self.server = None
        self.flush()

    def _on_request(self, ctx, method, path, body, blen, resp):
        try:
            m = method.decode()
            p = path.decode()
            data = ctypes.string_at(body, blen) if blen else b""
            status, ctype, out = self.handle(m, p, data)
        except Exception as e:
            status, ctype, out = 500, "application/json", json.dumps({"error": str(e)}).encode()
            self.last_error = traceback.format_exc()
        native.rt().dtr_http_respond(resp, status, ctype.encode(), out, len(out))

    # ─────────── routing (routes.rs:22-34) ───────────
    def handle(self, method: str, path: str, body: bytes) -> Tuple[int, str, bytes]:
        route = path.split("?", 1)[0]
        J = lambda s, o: (s, "application/json", json.dumps(o).encode())
        if method == "POST" and route == "/nodes/register":
            return J(*self.register(json.loads(body or b"{}")))
        if method == "POST" and route == "/delta":
            return J(*self.push_delta(json.loads(body)))
        if method == "PUT" and route.startswith("/upload/"):
            key = route[len("/upload/"):]
            try:
                self.store.put(key, body)
                return 200, "text/plain", b""
            except Exception:
                return 500, "text/plain", b""
        if method == "GET" and route.startswith("/download/"):
            key = route[len("/download/"):]
            try:
                return 200, "application/octet-stream", self.store.get(key)
            except Exception:
                return 404, "text/plain", f"Not found: {key}".encode()
        if method == "GET" and route == "/checkpoint/latest":
            return J(200, self.latest_checkpoint())
        if method == "GET" and route == "/config":
            return J(200, self.node_auto_config())
        if method == "GET" and route == "/status":
            return J(200, self.status())
        if method == "POST" and route == "/heartbeat":
            return J(200, self.heartbeat(json.loads(body)))
        if method == "GET" and route == "/health":
            return J(200, {"status": "ok"})
        if method == "GET" and route == "/metrics":
            return 200, "text/plain; version=0.0.4; charset=utf-8", self.metrics.render().encode()
        return 404, "text/plain", b"not found"

    # ─────────── handlers ───────────
    def register(self, req: dict):
        r = P.RegisterRequest.from_dict(req)
        node_id = r.node_id or f"node_{uuid.uuid4().hex}"
        api_key = str(uuid.uuid4())
        now = P.utcnow()
        reg = P.NodeRegistration(node_id=node_id, gpu_model=r.gpu_model, gpu_memory_gb=r.gpu_memory_gb,
                                 bandwidth_mbps=r.bandwidth_mbps, registered_at=now, status="Active",
                                 api_key_hash=hashlib.sha256(api_key.encode()).hexdigest(), last_seen=now)
        try:
            registry = self.store.get_json(P.node_registry_path())
        except Exception:
            registry = []
        registry.append(reg.to_dict())
        self.metrics.registered_nodes = len(registry)
        self.metrics.active_nodes = sum(1 for n in registry if n.get("status") == "Active")
        try:
            self.store.put_json(P.node_registry_path(), registry)
        except Exception:
            return 500, {"error": "Failed to save registration"}
        if r.hardware:
            hw = P.HardwareProfile.from_dict(r.hardware)
            with self.lock:
                self.acc.cs.node_profiles[node_id] = P.NodeProfile(
                    device_type=hw.device_type, vram_mb=hw.vram_mb, gpu_model=hw.gpu_model,
                    expected_round_time=hw.expected_round_time_secs, step_time_secs=hw.step_time_secs,
                    h_mini=hw.h_mini)
        endpoint = self.cfg.external_storage_endpoint or self.cfg.storage.endpoint
        resp = P.RegisterResponse(node_id=node_id, api_key=api_key, status="Active", storage_endpoint=endpoint,
                                  storage_bucket=self.cfg.storage.bucket,
                                  training_params=TrainingParams().to_dict())
        return 200, resp.to_dict()

    def push_delta(self, body: dict):
        push = P.DeltaPush.from_dict(body)
        self.metrics.delta_pushes_total += 1
        with self.lock:
            merging = self.acc.merging
            ok, reason = self.acc.push(push)
            current = self.acc.state.checkpoint_version
            n_contrib = len(self.acc.state.contributions)
            if ok and not merging:
                c = self.acc.state.contributions[-1]
                staleness = max(current - push.checkpoint_version, 0)
                self._append_stats({"event": "delta_accepted", "timestamp": P.to_rfc3339(P.utcnow()),
                                    "node_id": push.node_id, "seq_num": push.seq_num,
                                    "checkpoint_version": push.checkpoint_version, "inner_steps": push.inner_steps,
                                    "training_loss": push.training_loss, "weight": c.weight, "staleness": staleness,
                                    "tokens_processed": push.tokens_processed,
                                    **{k: v for k, v in (("compressed_bytes", push.compressed_bytes),
                                                         ("dense_norm", push.dense_norm),
                                                         ("sparse_norm", push.sparse_norm)) if v is not None}})
        if ok:
            self.metrics.delta_pushes_accepted += 1
        else:
            self.metrics.delta_pushes_rejected += 1
        self.metrics.accumulator_contributions = n_contrib
        self.maybe_aggregate()
        return 200, P.DeltaPushResponse(accepted=ok, checkpoint_version=current, reason=reason).to_dict()

    def latest_checkpoint(self):
        v = self.acc.state.checkpoint_version
        return P.CheckpointInfo(version=v, checkpoint_key=P.checkpoint_path(v),
                                metadata_key=P.checkpoint_metadata_path(v), val_loss=None, total_contributions=0,
                                total_tokens=0, created_at=P.to_rfc3339(P.utcnow())).to_dict()

    def node_auto_config(self):
        s = self.cfg.storage
        return {"storage": {"endpoint": self.cfg.external_storage_endpoint or s.endpoint, "bucket": s.bucket,
                            "access_key_id": s.access_key_id,
                            "secret_access_key": s.secret_access_key if self.cfg.publish_storage_secret else "",
                            "region": s.region},
                "training_params": TrainingParams().to_dict(), "coordinator_version": VERSION}

    def status(self):
        now = int(time.time())
        with self.lock:
            st, cs = self.acc.state, self.acc.cs
            active = sum(1 for ts in cs.heartbeats.values() if now - ts < 30 * 60)
            tw = sum(c.weight for c in st.contributions)
            avg = sum(c.training_loss * c.weight for c in st.contributions) / tw if tw > 0 else 0.0
            return P.TrainingStatus(checkpoint_version=st.checkpoint_version, active_nodes=active,
                                    total_contributions=st.version, total_tokens_trained=cs.total_tokens_trained,
                                    accumulator_contributions=len(st.contributions),
                                    latest_val_loss=avg if avg > 0 else None, loss_history=[],
                                    node_last_seen=[[k, v] for k, v in cs.heartbeats.items()]).to_dict()

    def heartbeat(self, body: dict):
        req = P.HeartbeatRequest.from_dict(body)
        now = int(time.time())
        with self.lock:
            cs = self.acc.cs
            cs.heartbeats[req.node_id] = now
            cs.heartbeats = {k: v for k, v in cs.heartbeats.items() if now - v < 10 * 60}
            cs.active_nodes = len(cs.heartbeats)
            active = cs.active_nodes
            cur = self.acc.state.checkpoint_version
        self.metrics.active_nodes = active
        abort = req.checkpoint_version is not None and max(cur - req.checkpoint_version, 0) >= 3
        return P.HeartbeatResponse(active_nodes=active, should_abort=abort, latest_version=cur).to_dict()

    # ─────────── stats JSONL (stats.rs:51-77, read-modify-write) ───────────
    def _save_outer_lr_state(self, outer_lr: float, delta_norm: float):
        """state/outer_lr.json: the applied outer lr and momentum and the last 10 merged-delta norms
        (the reference's OuterLrState, aggregation.rs:120-127, 214-218, 360-365)."""
        try:
            try:
                st = self.store.get_json(P.outer_lr_state_path())
            except Exception:
                st = {}
            norms = (list(st.get("recent_norms", [])) + [float(delta_norm)])[-10:]
            self.store.put_json(P.outer_lr_state_path(), {"outer_lr": outer_lr, "outer_momentum": 0.0,
                                                          "recent_norms": norms})
        except Exception as e:  # the reference only warns when this write fails
            log.warning("outer lr state not saved: %s", e)

    def _append_stats(self, entry: dict):
        try:
            try:
                cur = self.store.get(P.stats_history_path())
            except StorageError:
                cur = b""
            self.store.put(P.stats_history_path(), cur + (json.dumps(entry) + "\n").encode())
        except Exception:
            pass

    # ─────────── aggregation ───────────
    def maybe_aggregate(self, now=None, blocking: bool = False):
        with self.lock:
            if self.acc.merging or not self.acc.ready(now):
                return False
            snap = self.acc.begin_merge()
        self.metrics.aggregations_total += 1
        try:
            self.store.put_json(P.accumulator_path(), snap.to_dict())
        except Exception:
            pass
        t = threading.Thread(target=self._aggregate, args=(snap,), daemon=True)
        self.agg_thread = t
        t.start()
        if blocking:
            t.join()
        return True

    def _decode(self, data: bytes, shapes: Dict[str, list]) -> Dict[str, torch.Tensor]:
        if data[:4] == b"DTZ1" or (data[:4] == b"\x28\xb5\x2f\xfd" and native.zstd_decompress(data)[:4] == b"DTZ1"):
            flat = decode_dtz_dense(data)
            out, off = {}, 0
            for name in sorted(shapes):
                n = math.prod(shapes[name])
                out[name] = flat[off:off + n]
                off += n
            return out
        d = decode_delta(data)
        if isinstance(d, LowRankPayload):
            from ..parallel.lowrank import decompress_lowrank
            return decompress_lowrank(d)
        return d

    def _aggregate(self, snap: P.AccumulatorState):
        from ..utils.tracing import nvtx
        with nvtx("aggregate"):
            return self._aggregate_impl(snap)

    def _aggregate_impl(self, snap: P.AccumulatorState):
        t0 = time.time()
        try:
            new_version = snap.checkpoint_version + 1
            ck_bytes = self.store.get(P.checkpoint_path(snap.checkpoint_version))
            ckpt = load_safetensors_bytes(ck_bytes)
            shapes = {k: list(v.shape) for k, v in ckpt.items()}
            try:
                velocity = load_velocity(self.store.get(P.optimizer_state_path(snap.checkpoint_version)))
            except Exception:
                velocity = None
            deltas, weights, meta = [], [], []
            rejected = 0
            for c in snap.contributions:
                try:
                    d = self._decode(self.store.get(c.delta_key), shapes)
                    deltas.append({k: v.reshape(-1) for k, v in d.items()})
                    weights.append(c.weight)
                    meta.append(c)
                except Exception:
                    rejected += 1
            flat_ck = {k: v.reshape(-1).float() for k, v in ckpt.items()}
            dev = torch.device(self.merge_device)
            if dev.type != "cpu":
                flat_ck = {k: v.to(dev) for k, v in flat_ck.items()}
                deltas = [{k: v.to(dev) for k, v in d.items()} for d in deltas]
                if velocity is not None:
                    velocity = {k: v.to(dev) for k, v in velocity.items()}
            # outer lr: 1.0 once the contributions report a training loss, the configured initial value
            # before that; momentum 0 (aggregation.rs:141-144, 181-214, 364)
            lw = sum(c.weight for c in snap.contributions)
            avg_loss = sum(c.training_loss * c.weight for c in snap.contributions) / lw if lw > 0 else 0.0
            outer_lr = 1.0 if avg_loss > 0 else float(self.cfg.outer_lr)
            new, velocity, info = merge_reference(flat_ck, deltas, weights, velocity=velocity, outer_lr=outer_lr,
                                                  outer_momentum=0.0)
            rejected += info["rejected"]
            out = {k: new[k].reshape(shapes[k]).cpu() for k in new}
            self.store.put(P.checkpoint_path(new_version), save_safetensors(out))
            if velocity:
                self.store.put(P.optimizer_state_path(new_version),
                               save_velocity({k: v.cpu() for k, v in velocity.items()}))
            elapsed = time.time() - t0
            log.info("aggregation v%d: %d accepted, %d rejected, outer delta norm %.4g, %.2f s", new_version,
                     info["accepted"], rejected, info["outer_delta_norm"], elapsed)
            total_weight = sum(c.weight for c in snap.contributions)
            self.store.put_json(P.checkpoint_metadata_path(new_version), {
                "version": new_version, "contributions_accepted": info["accepted"], "contributions_rejected": rejected,
                "total_weight": total_weight, "outer_delta_norm": info["outer_delta_norm"],
                "aggregation_time_secs": elapsed, "outer_lr": outer_lr})
            self._save_outer_lr_state(outer_lr, info["outer_delta_norm"])
            st_hist: Dict[int, int] = {}
            for c in meta:
                s = max(snap.checkpoint_version - c.checkpoint_version, 0)
                st_hist[s] = st_hist.get(s, 0) + 1
            self._append_stats({"event": "checkpoint_produced", "timestamp": P.to_rfc3339(P.utcnow()),
                                "version": new_version, "contributions": info["accepted"],
                                "total_weight": total_weight, "outer_delta_norm": info["outer_delta_norm"],
                                "aggregation_time_secs": elapsed, "outer_lr": outer_lr,
                                "avg_loss": sum(c.training_loss for c in meta) / max(len(meta), 1),
                                "total_tokens": sum(c.tokens_processed for c in meta),
                                "staleness_histogram": sorted(st_hist.items()),
                                "per_delta_norms": info["per_delta_norms"]})
            tokens = sum(c.tokens_processed for c in snap.contributions)
            with self.lock:
                self.acc.finish_merge(new_version, [c.node_id for c in snap.contributions], tokens)
            self.metrics.checkpoint_version = new_version
            self.metrics.accumulator_contributions = len(self.acc.state.contributions)
            self.metrics.last_aggregation_secs = elapsed
            self.metrics.last_outer_delta_norm = info["outer_delta_norm"]
            self.flush()
            if new_version > self.cfg.keep_versions:
                threading.Thread(target=self._cleanup, args=(new_version - self.cfg.keep_versions,),
                                 daemon=True).start()
        except Exception:
            self.last_error = traceback.format_exc()
            self.metrics.aggregations_failed += 1
            with self.lock:
                self.acc.abort_merge()
        # contributions carried over from the merge window may already satisfy the trigger
        threading.Thread(target=self.maybe_aggregate, daemon=True).start()

    def _cleanup(self, up_to: int):
        for v in range(up_to):
            for k in (P.checkpoint_path(v), P.checkpoint_metadata_path(v), P.optimizer_state_path(v)):
                try:
                    self.store.delete(k)
                except Exception:
                    pass
            try:
                for k in self.store.list_keys(f"deltas/v{v}/"):
                    self.store.delete(k)
            except Exception:
                pass


def bootstrap(store: ObjectStore, model_cfg, seed: int = 0, init_std: float = 0.02, vocab_override=None,
              init_state=None):
    """Write checkpoint v0 + metadata + an empty accumulator (reference node/cli/src/main.rs:1247-1304).
    ``init_state``: start from these weights (e.g. an imported pretrained model) instead of a seeded init."""
    from ..models.params import ParamLayout, init_flat
    L = ParamLayout(model_cfg)
    if init_state is not None:
        flat = torch.zeros(L.total)
        L.load_state_dict(flat, init_state)
    else:
        flat = init_flat(L, init_std, seed)
    store.ensure_bucket()
    store.put(P.checkpoint_path(0), save_safetensors(L.to_state_dict(flat)))
    store.put_json(P.checkpoint_metadata_path(0), {"version": 0, "model_preset": "custom",
                                                   "param_count": L.num_params(), "bootstrap": True})
    store.put_json(P.accumulator_path(), P.AccumulatorState().to_dict())
    return L, flat
