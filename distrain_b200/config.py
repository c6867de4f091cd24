"""Typed configuration: model presets, training/compression parameters, coordinator and node configs.

Field names and defaults follow the reference so JSON/TOML written by either side loads in the other:

* ``ModelConfig`` / presets:           core/model/src/config.rs:9-160
* ``TrainingParams``:                  core/shared/src/types.rs:144-191
* ``CompressionConfig``:               core/model/src/compression.rs:31-53
* ``StorageConfig/CoordinatorConfig``: core/shared/src/config.rs:8-78
* ``NodeConfig``:                      core/shared/src/config.rs:81-143

Presets keep the reference values (micro: vocab 256, seq 64, theta 5e5; all others theta 5e5).
``bench_config`` returns the benchmark workloads (micro-test at vocab 32768 / seq 128 / theta 1e4,
tiny 1024x32, small 2048x8, large TP=2 2048x4) as explicit overrides on top of the presets.
"""
from __future__ import annotations

import dataclasses
import json
import math
import os
from dataclasses import dataclass, field, asdict, fields
from typing import Any, Dict, Optional


def _from_dict(cls, d: Dict[str, Any]):
    """Build dataclass ``cls`` from a dict, ignoring unknown keys and keeping defaults for missing ones."""
    import typing
    hints = typing.get_type_hints(cls)
    names = {f.name for f in fields(cls)}
    kw = {}
    for k, v in d.items():
        if k not in names:
            continue
        t = hints.get(k)
        if dataclasses.is_dataclass(t) and isinstance(v, dict):
            v = _from_dict(t, v)
        kw[k] = v
    return cls(**kw)


class _Json:
    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)

    def to_json(self) -> str:
        return json.dumps(self.to_dict())

    @classmethod
    def from_dict(cls, d: Dict[str, Any]):
        return _from_dict(cls, d)

    @classmethod
    def from_json(cls, s: str):
        return cls.from_dict(json.loads(s))


# ─────────────────────────────────────────────────────────────────────────────
# Model
# ─────────────────────────────────────────────────────────────────────────────
@dataclass
class ModelConfig(_Json):
    hidden_dim: int = 768
    num_layers: int = 12
    num_heads: int = 12
    num_kv_heads: int = 4
    vocab_size: int = 32768
    max_seq_len: int = 4096
    ffn_hidden_dim: int = 2048
    rope_theta: float = 500_000.0
    norm_eps: float = 1e-5
    qkv_bias: bool = True
    attention_dropout: float = 0.0
    tie_embeddings: bool = True

    def head_dim(self) -> int:
        return self.hidden_dim // self.num_heads

    def num_gqa_groups(self) -> int:
        assert self.num_heads % self.num_kv_heads == 0
        return self.num_heads // self.num_kv_heads

    def kv_dim(self) -> int:
        return self.head_dim() * self.num_kv_heads

    def param_count(self) -> int:
        """Same formula as the reference's ``param_count`` (core/model/src/config.rs:35-57)."""
        emb = self.vocab_size * self.hidden_dim
        kv = self.kv_dim()
        attn = self.hidden_dim * self.hidden_dim * 2 + self.hidden_dim * kv * 2
        if self.qkv_bias:
            attn += self.hidden_dim + 2 * kv
        ffn = 3 * self.hidden_dim * self.ffn_hidden_dim
        block = attn + ffn + 2 * self.hidden_dim
        total = emb + self.num_layers * block + self.hidden_dim
        if not self.tie_embeddings:
            total += emb
        return total

    def flops_per_token(self, seq_len: int) -> float:
        """Training FLOPs per token: 6 x matmul params (incl. tied LM head) + causal attention."""
        h, f, kv = self.hidden_dim, self.ffn_hidden_dim, self.kv_dim()
        per_layer = h * (h + 2 * kv) + h * h + 3 * h * f
        dense = self.num_layers * per_layer + self.vocab_size * h
        attn = self.num_layers * 2 * 2 * seq_len * h / 2  # QK^T and PV, causal half
        return 6.0 * dense + 3.0 * attn


def _preset(h, l, nh, nkv, f, vocab=32768, seq=4096) -> ModelConfig:
    return ModelConfig(hidden_dim=h, num_layers=l, num_heads=nh, num_kv_heads=nkv,
                       ffn_hidden_dim=f, vocab_size=vocab, max_seq_len=seq)


# Reference preset table (core/model/src/config.rs:61-149).
PRESETS: Dict[str, ModelConfig] = {
    "micro": _preset(64, 2, 4, 2, 128, vocab=256, seq=64),
    "tiny": _preset(768, 12, 12, 4, 2048),
    "small": _preset(2048, 24, 16, 4, 5504),
    "medium": _preset(4096, 32, 32, 8, 11008),
    "large": _preset(5120, 40, 40, 8, 13824),
}
# Reference aliases (config.rs:151-160).
_ALIASES = {"micro": "micro", "micro-test": "micro", "125m": "tiny", "tiny": "tiny",
            "1b": "small", "small": "small", "7b": "medium", "medium": "medium",
            "13b": "large", "large": "large"}


def preset(name: str) -> ModelConfig:
    key = _ALIASES.get(name)
    if key is None:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(_ALIASES)}")
    return dataclasses.replace(PRESETS[key])


# ─────────────────────────────────────────────────────────────────────────────
# Training / compression
# ─────────────────────────────────────────────────────────────────────────────
@dataclass
class TrainingParams(_Json):
    """Canonical training hyper-parameters handed out by the coordinator (types.rs:144-191)."""
    batch_size: int = 4
    seq_len: int = 512
    lr_max: float = 3e-4
    lr_min: float = 1e-6
    weight_decay: float = 0.1
    grad_clip_norm: float = 1.0
    warmup_fraction: float = 0.2
    shards_fraction: float = 0.2
    min_inner_steps: int = 50
    max_inner_steps: int = 500
    target_push_interval_secs: float = 60.0

    def shards_per_node(self, total_shards: int) -> int:
        return min(max(int(total_shards * self.shards_fraction), 2), total_shards)


@dataclass
class CompressionConfig(_Json):
    """Delta compression settings (compression.rs:31-53) plus the block-INT8 extension.

    ``int8_block`` = 0 reproduces the reference's per-tensor absmax/127 scale; > 0 gives one fp32
    absmax scale per ``int8_block`` kept values (block 256 in the benchmark configs).
    """
    top_k_fraction: float = 0.01
    quantize_int8: bool = True
    zstd_level: int = 3
    min_top_k_fraction: float = 0.001
    max_top_k_fraction: float = 0.1
    per_tensor_adaptive: bool = True
    int8_block: int = 256

    def reference_dict(self) -> Dict[str, Any]:
        """The reference's JSON shape of this struct (no ``int8_block``)."""
        d = self.to_dict()
        d.pop("int8_block")
        return d


@dataclass
class OptimConfig(_Json):
    """Inner AdamW. betas/eps are the defaults of the reference's optimizer (Burn ``AdamWConfig``);
    clipping is per-parameter-tensor L2 norm (Burn ``GradientClipping::Norm``) unless ``clip_global``."""
    lr: float = 3e-4
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-5
    weight_decay: float = 0.1
    grad_clip_norm: float = 1.0
    clip_global: bool = False
    # Reference scales lr linearly with batch/4 (node/cli/src/continuous.rs:419-424); off by default.
    lr_batch_scaling: bool = False
    warmup_fraction: float = 0.2


# ─────────────────────────────────────────────────────────────────────────────
# Services
# ─────────────────────────────────────────────────────────────────────────────
DEFAULT_BUCKET = "distrain-training"


@dataclass
class StorageConfig(_Json):
    endpoint: str = "http://localhost:9000"
    bucket: str = DEFAULT_BUCKET
    access_key_id: str = "minioadmin"
    secret_access_key: str = "minioadmin"
    region: str = "auto"


@dataclass
class CoordinatorConfig(_Json):
    host: str = "0.0.0.0"
    port: int = 8000
    storage: StorageConfig = field(default_factory=StorageConfig)
    min_contributions: int = 4
    staleness_decay: float = 0.9
    max_staleness: int = 10
    outer_lr: float = 0.1
    outer_momentum: float = 0.9
    keep_versions: int = 10
    vocab_size: int = 32768
    min_weight: float = 1.5
    max_storage_gb: int = 0
    external_storage_endpoint: Optional[str] = None
    # GET /config hands nodes the object-store credentials, secret included, as the reference does
    # (routes.rs:423-444); False withholds the secret for deployments whose nodes carry their own
    publish_storage_secret: bool = True

    @classmethod
    def from_env(cls, env: Optional[Dict[str, str]] = None) -> "CoordinatorConfig":
        """Environment mapping of the reference (coordinator/src/main.rs:141-188)."""
        e = dict(os.environ if env is None else env)
        c = cls()
        c.host = e.get("HOST", c.host)
        c.port = int(e.get("PORT", c.port))
        c.storage = StorageConfig(
            endpoint=e.get("R2_ENDPOINT", c.storage.endpoint),
            bucket=e.get("R2_BUCKET", c.storage.bucket),
            access_key_id=e.get("R2_ACCESS_KEY_ID", c.storage.access_key_id),
            secret_access_key=e.get("R2_SECRET_ACCESS_KEY", c.storage.secret_access_key),
            region=e.get("R2_REGION", c.storage.region))
        for name, conv in (("MIN_CONTRIBUTIONS", int), ("OUTER_LR", float), ("OUTER_MOMENTUM", float),
                           ("KEEP_VERSIONS", int), ("MAX_STALENESS", int), ("VOCAB_SIZE", int),
                           ("MIN_WEIGHT", float)):
            if name in e:
                setattr(c, name.lower(), conv(e[name]))
        if "STALENESS_DECAY" in e:
            c.staleness_decay = float(e["STALENESS_DECAY"])
        if e.get("S3_EXTERNAL_ENDPOINT"):
            c.external_storage_endpoint = e["S3_EXTERNAL_ENDPOINT"]
        if "PUBLISH_STORAGE_SECRET" in e:
            c.publish_storage_secret = e["PUBLISH_STORAGE_SECRET"].strip().lower() not in ("0", "false", "no")
        return c


@dataclass
class NodeConfig(_Json):
    coordinator_url: str = "http://localhost:8000"
    api_key: str = ""
    storage: StorageConfig = field(default_factory=StorageConfig)
    gpu_device: int = -1
    target_push_interval_secs: float = 60.0
    min_inner_steps: int = 10
    max_inner_steps: int = 500
    cache_dir: str = "~/.distrain/cache"
    max_cache_gb: int = 100
    batch_size: Optional[int] = None
    seq_len: int = 512
    training_params: Optional[Dict[str, Any]] = None
    max_memory_fraction: float = 0.80
    force_batch_size: Optional[int] = None
    force_cpu: bool = False

    @classmethod
    def load_toml(cls, path: str) -> "NodeConfig":
        import tomllib
        with open(path, "rb") as f:
            return cls.from_dict(tomllib.load(f))


# ─────────────────────────────────────────────────────────────────────────────
# Benchmark workloads
# ─────────────────────────────────────────────────────────────────────────────
@dataclass
class RunConfig(_Json):
    """One training workload: model + batch geometry + inner/outer optimisation + compression."""
    name: str = "tiny"
    model: ModelConfig = field(default_factory=lambda: preset("tiny"))
    seq_len: int = 1024
    micro_batch: int = 32
    # micro-batches per optimizer step: gradients of grad_accum_steps x micro_batch sequences are summed
    # before one clip + AdamW update (the effective batch); push_every counts optimizer steps
    grad_accum_steps: int = 1
    push_every: int = 50
    optim: OptimConfig = field(default_factory=OptimConfig)
    compression: CompressionConfig = field(default_factory=lambda: CompressionConfig(
        top_k_fraction=0.10, quantize_int8=True, per_tensor_adaptive=True, int8_block=256))
    bandwidth_adaptive: bool = False
    tp: int = 1
    activation_checkpointing: bool = False
    outer_lr: float = 1.0
    staleness_decay: float = 0.9
    max_staleness: int = 10
    init_std: float = 0.02
    seed: int = 0
    # What a node does at a checkpoint swap. The reference node (continuous.rs:458-502) pushes the steps
    # trained since its last push as a partial round, replaces its weights with the checkpoint, keeps
    # its error-feedback buffer and re-creates AdamW: swap_mode="push_partial", ef_on_swap="keep",
    # reset_optimizer_on_swap=True. On one box a merge lands within a step or two of the pushes, so that
    # turns every push into a cascade of few-step partial rounds and optimizer restarts. The defaults
    # here, chosen on the held-out loss at matched tokens (2 nodes x 300 steps of the tiny preset on a
    # learnable Markov source: 1.67 against 2.35 for the reference's choices; dense NCCL averaging
    # 1.67 with optimizer restarts, 1.55 without):
    #   swap_mode "rebase": carry the steps since the last push onto the checkpoint
    #     (weights = checkpoint + (weights - round start)) and keep the round going, so every push
    #     covers push_every steps;
    #   ef_on_swap "fold": clear the error-feedback buffer at the boundary by moving its residual into
    #     the weights (weights -= residual); the next delta transmits it, while the node trains on all
    #     of its own progress ("keep" and "reset" are the other choices);
    #   reset_optimizer_on_swap False: keep the AdamW moments.
    payload_slots: int = 2  # compressed-delta buffers per node (1 halves that memory; pushes then wait for the merge)
    # in-box checkpoint persistence: object-store directory ("" = off), every N versions, newest kept; resume
    # starts every node from the newest stored version
    checkpoint_store: str = ""
    checkpoint_every: int = 0
    keep_versions: int = 10
    resume: bool = False
    metrics_port: int = -1  # in-box coordinator's Prometheus /metrics (-1 = off, 0 = any free port)
    # SMs of the green-context partition every GPU's merge kernels run in (the driver rounds up to its
    # granularity, 8 on this architecture); training keeps the whole GPU and the merge never takes more
    # than the partition. 0 = a top-priority stream over the whole device
    merge_sms: int = 16
    # inner lr: constant (default) or loss-based, lr_max * clamp(loss_ema / ln(vocab), 0.1, 1)
    # (reference continuous.rs:586-596, LR_MODE=loss_based)
    loss_based_lr: bool = False
    # per-step watchdog: expected seconds per step (0 = off); a step stalled past max(6x, 300 s) is reported
    watchdog_step_secs: float = 0.0
    swap_mode: str = "rebase"
    ef_on_swap: str = "fold"
    reset_optimizer_on_swap: bool = False


def bench_config(name: str) -> RunConfig:
    """Named benchmark workloads (micro-test CPU, tiny 8x1, small 8x1, large TP=2)."""
    if name in ("micro", "micro-test"):
        m = preset("micro")
        m.vocab_size, m.max_seq_len, m.rope_theta = 32768, 128, 10000.0
        return RunConfig(name="micro-test", model=m, seq_len=128, micro_batch=4, push_every=20,
                         compression=CompressionConfig(top_k_fraction=0.10, int8_block=256))
    if name in ("tiny", "125m"):
        return RunConfig(name="tiny", model=preset("tiny"), seq_len=1024, micro_batch=32, push_every=50)
    if name in ("small", "1b"):
        return RunConfig(name="small", model=preset("small"), seq_len=2048, micro_batch=8, push_every=100,
                         bandwidth_adaptive=True,
                         compression=CompressionConfig(top_k_fraction=0.99, int8_block=256))
    if name in ("large", "13b"):
        return RunConfig(name="large", model=preset("large"), seq_len=2048, micro_batch=4, push_every=100,
                         tp=2, activation_checkpointing=True, payload_slots=1)
    if name in ("medium", "7b"):
        # 5.8 B parameters: with the protocol's buffers one GPU would need ~192 GB, so two GPUs per node
        return RunConfig(name="medium", model=preset("medium"), seq_len=2048, micro_batch=4, push_every=100,
                         tp=2, activation_checkpointing=True, payload_slots=1)
    raise KeyError(name)


def cosine_lr(step: int, warmup_steps: int, total_steps: int, max_lr: float, min_lr: float) -> float:
    """Linear warmup then cosine decay, same argument order and formula as the reference
    (core/model/src/training.rs:282-289; no clamp past ``total_steps``)."""
    if step < warmup_steps:
        return max_lr * (step / warmup_steps)
    progress = (step - warmup_steps) / max(total_steps - warmup_steps, 1)
    return min_lr + 0.5 * (max_lr - min_lr) * (1.0 + math.cos(math.pi * progress))
