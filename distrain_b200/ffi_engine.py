"""Engine state behind the C ABI of ``libdistrain_c.so`` (``csrc/ffi/distrain_c.cpp``).

One model with its optimizer, a token source, a parameter snapshot and an error-feedback buffer,
driven by calls that take plain values and return JSON text. The C library forwards every
``distrain_*`` call to the method of the same name here. This is the counterpart of the reference's
FFI engine (node/ffi/src/lib.rs:79-582): the same function set, argument order and JSON replies
(StatusResponse, StepResult, CalibrationResult, ``{"error": ...}``), so a C, Swift or Kotlin caller
written against it can switch. Two things differ on purpose:

* the AdamW optimizer (weight decay 0.1, gradient clipping 1.0) keeps its moments from step to step;
  the reference creates a new one inside every ``distrain_train_step`` (lib.rs:338-345), so its steps
  are plain clipped sign-like updates with no history;
* the GPU backend is the sm_100a ``TrainEngine`` (bf16 compute, fp32 master); the CPU backend is the
  fp32 oracle model with the same optimizer semantics.
"""
from __future__ import annotations

import functools
import json
import time
from typing import Dict, Optional

import torch

PRESETS = {"microtest": "micro", "micro": "micro", "micro-test": "micro", "tiny": "tiny", "small": "small",
           "medium": "medium", "large": "large"}


def _reply(fn):
    @functools.wraps(fn)
    def wrapped(self, *a):
        try:
            return json.dumps(fn(self, *a))
        except Exception as e:  # every failure reaches the C caller as {"error": ...}
            return json.dumps({"error": f"{type(e).__name__}: {e}"})
    return wrapped


class FfiEngine:
    def __init__(self):
        self.use_gpu = True
        self._clear()

    def _clear(self):
        self.cfg = None
        self.preset = "none"
        self.backend = None
        self.params: Optional[Dict[str, torch.Tensor]] = None  # weights while no backend holds them
        self.loader = None
        self.batch = self.seq = None
        self.step = 0
        self.last_loss = 0.0
        self.total_tokens = 0
        self.snapshot: Optional[Dict[str, torch.Tensor]] = None
        self.ef: Dict[str, torch.Tensor] = {}

    # ── backend ──
    def _gpu(self) -> bool:
        return bool(self.use_gpu) and torch.cuda.is_available()

    def _state(self) -> Dict[str, torch.Tensor]:
        if self.backend is not None:
            return {k: v.detach().float().cpu().clone() for k, v in self.backend.state().items()}
        return {k: v.clone() for k, v in self.params.items()}

    def _make_backend(self, state):
        from .config import OptimConfig
        from .parallel.http_node import CpuBackend, CudaBackend
        if self._gpu():
            self.backend = CudaBackend(self.cfg, OptimConfig(), self.batch, self.seq, torch.device("cuda", 0))
        else:
            self.backend = CpuBackend(self.cfg, OptimConfig())
        self.backend.load(state)
        self.params = None

    def _load(self, cfg, sd, preset: str, keep_ef: bool):
        """New weights: the data source stays; the error-feedback residual stays across a checkpoint
        load (it belongs to the node, not to one checkpoint) and is dropped by a fresh init."""
        loader, batch, seq, ef = self.loader, self.batch, self.seq, self.ef
        self._clear()
        self.loader, self.batch, self.seq = loader, batch, seq
        if keep_ef:
            self.ef = ef
        self.cfg, self.preset = cfg, preset
        self.params = {k: v.detach().float().clone() for k, v in sd.items()}
        if self.loader is not None:
            self.cfg.max_seq_len = max(self.cfg.max_seq_len, self.seq)

    def _require(self):
        if self.cfg is None:
            raise RuntimeError("engine not initialised: call distrain_init or distrain_load_checkpoint first")

    # ── the C ABI ──
    def set_backend(self, use_gpu: int):
        self.use_gpu = bool(use_gpu)
        return json.dumps({"ok": True, "gpu": self._gpu()})

    @_reply
    def init(self, preset_json: str):
        from .config import preset
        from .models.params import ParamLayout, init_flat
        name = preset_json.strip().strip('"')
        key = PRESETS.get(name.lower())
        if key is None:
            raise ValueError(f"unknown preset: {name}")
        cfg = preset(key)
        L = ParamLayout(cfg)
        self._load(cfg, L.to_state_dict(init_flat(L, 0.02, 0)), name, keep_ef=False)
        return self._status()

    @_reply
    def load_shards(self, paths_json: str, batch_size: int, seq_len: int):
        from .utils.data import ShardLoader
        paths = json.loads(paths_json)
        if not isinstance(paths, list) or not paths:
            raise ValueError("paths_json must be a non-empty JSON array of shard paths")
        if batch_size < 1 or seq_len < 2:
            raise ValueError("batch_size >= 1 and seq_len >= 2 are required")
        self.loader = ShardLoader([str(p) for p in paths], int(seq_len), int(batch_size))
        from .parallel.http_node import CudaBackend
        if (self.batch, self.seq) != (batch_size, seq_len) and isinstance(self.backend, CudaBackend):
            state = self._state()  # the GPU engine is built for one batch shape (the CPU model is not)
            self.backend = None
            self.params = state
        self.batch, self.seq = int(batch_size), int(seq_len)
        if self.cfg is not None:
            self.cfg.max_seq_len = max(self.cfg.max_seq_len, self.seq)
        return {"ok": True, "shards": len(paths)}

    @_reply
    def train_step(self, learning_rate: float):
        self._require()
        if self.loader is None:
            raise RuntimeError("no data loaded: call distrain_load_shards first")
        if self.backend is None:
            self._make_backend(self.params)
        tokens = self.loader.next_batch()
        loss = self.backend.step(tokens, float(learning_rate))
        self.step += 1
        self.last_loss = loss
        self.total_tokens += self.batch * self.seq
        return {"loss": loss, "step": self.step, "tokens_processed": self.total_tokens}

    def _status(self):
        return {"initialized": self.cfg is not None, "step": self.step, "last_loss": self.last_loss,
                "total_tokens": self.total_tokens, "model_preset": self.preset, "gpu": self._gpu()}

    @_reply
    def status(self):
        return self._status()

    @_reply
    def calibrate(self, target_interval_secs: float):
        """Seconds per training step of this model on this device, timed on a throwaway copy (batch 1,
        synthetic tokens, 5 steps after one warm-up), and the steps per push that fill the target
        interval, within [5, 1000] (the reference's rule, node/ffi/src/lib.rs:379-400)."""
        from .config import OptimConfig, preset
        from .models.params import ParamLayout, init_flat
        from .parallel.http_node import CpuBackend, CudaBackend
        cfg = self.cfg if self.cfg is not None else preset("micro")
        gpu = self._gpu()
        seq = 129 if gpu else min(cfg.max_seq_len, 33)
        L = ParamLayout(cfg)
        sd = L.to_state_dict(init_flat(L, 0.02, 1))
        if gpu:
            b = CudaBackend(cfg, OptimConfig(), 1, seq, torch.device("cuda", 0))
        else:
            b = CpuBackend(cfg, OptimConfig())
        b.load(sd)
        g = torch.Generator().manual_seed(0)
        toks = [torch.randint(0, cfg.vocab_size, (1, seq), generator=g, dtype=torch.int32) for _ in range(6)]
        b.step(toks[0], 1e-4)
        steps = 5
        t0 = time.perf_counter()
        for t in toks[1:]:
            b.step(t, 1e-4)
        secs = (time.perf_counter() - t0) / steps
        del b
        h = int(float(target_interval_secs) / max(secs, 1e-9))
        return {"secs_per_step": secs, "recommended_h_mini": max(5, min(1000, h))}

    @_reply
    def load_checkpoint(self, data: bytes):
        from .utils.checkpoint import load_safetensors_bytes
        if not data:
            raise ValueError("null or empty checkpoint data")
        return self._load_ckpt(load_safetensors_bytes(bytes(data)))

    @_reply
    def load_checkpoint_file(self, path: str):
        from .utils.checkpoint import load_safetensors
        return self._load_ckpt(load_safetensors(path))

    def _load_ckpt(self, sd):
        from .cli import _infer_model_config
        cfg = _infer_model_config(sd)
        self._load(cfg, sd, "checkpoint", keep_ef=True)
        n = sum(v.numel() for v in sd.values())
        return {"ok": True, "num_params": n, "max_seq_len": cfg.max_seq_len, "gpu": self._gpu()}

    @_reply
    def snapshot_params(self):
        self._require()
        self.snapshot = self._state()
        return {"ok": True, "num_params": sum(v.numel() for v in self.snapshot.values())}

    @_reply
    def compute_delta(self, output_path: str):
        """Delta = snapshot - current weights, compressed with the reference's default settings (error
        feedback, adaptive top-k 1 %, per-tensor INT8) into its zstd JSON format, written to a file."""
        from .config import CompressionConfig
        from .parallel.compression import compress_reference
        from .utils.delta_codec import encode_sparse_delta
        self._require()
        if self.snapshot is None:
            raise RuntimeError("no snapshot: call distrain_snapshot_params first")
        cur = self._state()
        delta = {k: self.snapshot[k] - cur[k] for k in self.snapshot}
        shapes = {k: list(v.shape) for k, v in cur.items()}
        sd, _ = compress_reference(delta, shapes, CompressionConfig(int8_block=0), self.ef)
        blob = encode_sparse_delta(sd)
        with open(output_path, "wb") as f:
            f.write(blob)
        return {"ok": True, "size_bytes": len(blob)}

    @_reply
    def default_training_params(self):
        from .config import TrainingParams
        return TrainingParams().to_dict()

    def shutdown(self):
        loader = self.loader
        self._clear()
        if loader is not None:
            loader.close()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
        return json.dumps({"ok": True})
