"""Node <-> coordinator protocol: wire types, storage key layout, accumulator and checkpoint trigger.

JSON shapes follow the reference's serde types field for field so either side can talk to the other:
  wire types          core/shared/src/types.rs:1-303   (NodeId newtype -> plain string, DateTime -> RFC3339)
  key layout          core/shared/src/paths.rs:3-51
  accumulator         coordinator/src/state.rs:63-124  (staleness reject, per-node replace by seq_num,
                                                        weight = tokens * decay^staleness)
  checkpoint trigger  coordinator/src/state.rs:140-225 (min contributions, all-active, patience window)
  node profiles       coordinator/src/state.rs:229-265

Differences from the reference (deliberate): contributions that arrive while a merge is running are
kept and re-weighted against the new version instead of being wiped by the post-merge reset
(routes.rs:338-346); see ``Accumulator.carry_over``.
"""
from __future__ import annotations

import datetime as _dt
import math
import time
from dataclasses import dataclass, field, asdict
from typing import Any, Dict, List, Optional, Tuple

from .config import _Json


# ─────────────────────────────── time helpers ───────────────────────────────
def utcnow() -> _dt.datetime:
    return _dt.datetime.now(_dt.timezone.utc)


def to_rfc3339(t: Optional[_dt.datetime]) -> Optional[str]:
    if t is None:
        return None
    return t.astimezone(_dt.timezone.utc).strftime("%Y-%m-%dT%H:%M:%S.%fZ")


def from_rfc3339(s: Optional[str]) -> Optional[_dt.datetime]:
    if s is None:
        return None
    s = s.strip()
    if s.endswith("Z"):
        s = s[:-1] + "+00:00"
    # chrono may emit nanoseconds; Python parses at most microseconds
    if "." in s:
        head, rest = s.split(".", 1)
        frac, tz = rest, ""
        for sep in ("+", "-"):
            if sep in rest:
                frac, tz = rest.split(sep, 1)
                tz = sep + tz
                break
        s = f"{head}.{frac[:6].ljust(6, '0')}{tz}"
    return _dt.datetime.fromisoformat(s)


# ─────────────────────────────── key layout ───────────────────────────────
DEFAULT_BUCKET = "distrain-training"


def checkpoint_path(version: int) -> str:
    return f"checkpoints/v{version}/model.safetensors"


def checkpoint_metadata_path(version: int) -> str:
    return f"checkpoints/v{version}/metadata.json"


def optimizer_state_path(version: int) -> str:
    return f"optimizer_state/v{version}/velocity.safetensors"


def delta_path(version: int, node_id: str, seq_num: int) -> str:
    return f"deltas/v{version}/{node_id}_{seq_num}.delta.zst"


def accumulator_path() -> str:
    return "accumulator/current.json"


def data_shard_path(shard_id: int) -> str:
    return f"data/shard_{shard_id:04d}.bin"


def manifest_path() -> str:
    return "data/manifest.json"


def run_config_path() -> str:
    return "config/run_config.json"


def node_registry_path() -> str:
    return "state/node_registry.json"


def outer_lr_state_path() -> str:
    return "state/outer_lr.json"


def stats_history_path() -> str:
    return "stats/training_history.jsonl"


def coordinator_state_path() -> str:
    return "state/coordinator.json"


# ─────────────────────────────── wire types ───────────────────────────────
@dataclass
class DeltaPush(_Json):
    node_id: str
    seq_num: int
    checkpoint_version: int
    inner_steps: int
    delta_key: str
    training_loss: float
    tokens_processed: int
    training_time_secs: float
    compressed_bytes: Optional[int] = None
    dense_norm: Optional[float] = None
    sparse_norm: Optional[float] = None


@dataclass
class DeltaPushResponse(_Json):
    accepted: bool
    checkpoint_version: int
    reason: Optional[str] = None

    def to_dict(self):
        d = asdict(self)
        if d["reason"] is None:  # serde skip_serializing_if = "Option::is_none"
            d.pop("reason")
        return d


@dataclass
class CheckpointInfo(_Json):
    version: int
    checkpoint_key: str
    metadata_key: str
    val_loss: Optional[float]
    total_contributions: int
    total_tokens: int
    created_at: str


@dataclass
class ContributionMeta:
    node_id: str
    seq_num: int
    weight: float
    checkpoint_version: int
    inner_steps: int
    tokens_processed: int
    delta_key: str
    received_at: _dt.datetime
    training_loss: float = 0.0

    def to_dict(self):
        d = asdict(self)
        d["received_at"] = to_rfc3339(self.received_at)
        return d

    @classmethod
    def from_dict(cls, d):
        d = dict(d)
        d["received_at"] = from_rfc3339(d["received_at"])
        d.setdefault("tokens_processed", 0)
        d.setdefault("training_loss", 0.0)
        return cls(**{k: d[k] for k in cls.__dataclass_fields__})


@dataclass
class AccumulatorState:
    checkpoint_version: int = 0
    contributions: List[ContributionMeta] = field(default_factory=list)
    version: int = 0
    first_contribution_at: Optional[_dt.datetime] = None

    def to_dict(self):
        return {"checkpoint_version": self.checkpoint_version,
                "contributions": [c.to_dict() for c in self.contributions],
                "version": self.version,
                "first_contribution_at": to_rfc3339(self.first_contribution_at)}

    @classmethod
    def from_dict(cls, d):
        return cls(checkpoint_version=d.get("checkpoint_version", 0),
                   contributions=[ContributionMeta.from_dict(c) for c in d.get("contributions", [])],
                   version=d.get("version", 0),
                   first_contribution_at=from_rfc3339(d.get("first_contribution_at")))


@dataclass
class TrainingStatus(_Json):
    checkpoint_version: int
    active_nodes: int
    total_contributions: int
    total_tokens_trained: int
    accumulator_contributions: int
    latest_val_loss: Optional[float]
    loss_history: List[Tuple[int, float]]
    node_last_seen: List[Tuple[str, int]] = field(default_factory=list)


@dataclass
class HeartbeatRequest(_Json):
    node_id: str
    step: Optional[int] = None
    total_steps: Optional[int] = None
    loss: Optional[float] = None
    checkpoint_version: Optional[int] = None


@dataclass
class HeartbeatResponse(_Json):
    active_nodes: int
    should_abort: bool = False
    latest_version: Optional[int] = None


DEVICE_TYPES = ("DiscreteGpu", "IntegratedGpu", "Cpu", "Unknown")
NODE_STATUSES = ("Pending", "Active", "Suspended", "Offline")


@dataclass
class HardwareProfile(_Json):
    gpu_model: str = ""
    vram_mb: int = 0
    device_type: str = "Unknown"
    cpu_cores: int = 0
    ram_mb: int = 0
    step_time_secs: Optional[float] = None
    h_mini: Optional[int] = None
    batch_size: Optional[int] = None
    expected_round_time_secs: Optional[float] = None


@dataclass
class RegisterRequest(_Json):
    gpu_model: str
    gpu_memory_gb: float
    bandwidth_mbps: float
    node_id: Optional[str] = None
    hardware: Optional[Dict[str, Any]] = None


@dataclass
class RegisterResponse(_Json):
    node_id: str
    api_key: str
    status: str
    storage_endpoint: Optional[str] = None
    storage_bucket: Optional[str] = None
    training_params: Optional[Dict[str, Any]] = None


@dataclass
class NodeRegistration:
    node_id: str
    gpu_model: str
    gpu_memory_gb: float
    bandwidth_mbps: float
    registered_at: _dt.datetime
    status: str
    api_key_hash: str
    last_seen: _dt.datetime
    total_contributions: int = 0

    def to_dict(self):
        d = asdict(self)
        d["registered_at"] = to_rfc3339(self.registered_at)
        d["last_seen"] = to_rfc3339(self.last_seen)
        return d

    @classmethod
    def from_dict(cls, d):
        d = dict(d)
        d["registered_at"] = from_rfc3339(d["registered_at"])
        d["last_seen"] = from_rfc3339(d["last_seen"])
        return cls(**{k: d[k] for k in cls.__dataclass_fields__ if k in d})


@dataclass
class NodeProfile:
    device_type: str = "Unknown"
    vram_mb: int = 0
    gpu_model: str = ""
    round_time_secs: Optional[float] = None
    expected_round_time: Optional[float] = None
    step_time_secs: Optional[float] = None
    h_mini: Optional[int] = None
    last_push_time: Optional[int] = None


@dataclass
class CoordinatorPersistentState:
    total_tokens_trained: int = 0
    active_nodes: int = 0
    recent_contributors: List[Tuple[int, List[str]]] = field(default_factory=list)
    heartbeats: Dict[str, int] = field(default_factory=dict)
    node_profiles: Dict[str, NodeProfile] = field(default_factory=dict)

    def to_dict(self):
        return {"total_tokens_trained": self.total_tokens_trained, "active_nodes": self.active_nodes,
                "recent_contributors": [[v, list(n)] for v, n in self.recent_contributors],
                "heartbeats": dict(self.heartbeats),
                "node_profiles": {k: asdict(v) for k, v in self.node_profiles.items()}}

    @classmethod
    def from_dict(cls, d):
        return cls(total_tokens_trained=d.get("total_tokens_trained", 0), active_nodes=d.get("active_nodes", 0),
                   recent_contributors=[(int(v), list(n)) for v, n in d.get("recent_contributors", [])],
                   heartbeats={k: int(v) for k, v in d.get("heartbeats", {}).items()},
                   node_profiles={k: NodeProfile(**v) for k, v in d.get("node_profiles", {}).items()})


# ─────────────────────────────── accumulator logic ───────────────────────────────
def _cstrs(items):
    import ctypes
    arr = (ctypes.c_char_p * max(len(items), 1))(*[x.encode() for x in items])
    return arr


def apply_delta_push(acc: AccumulatorState, push: DeltaPush, staleness_decay: float, max_staleness: int,
                     now: Optional[_dt.datetime] = None):
    """Returns (accepted, reason). The decision (staleness cap, dedup by seq_num, weight
    tokens * decay^staleness; reference state.rs:63-124) is the runtime library's ``dts_accept_push``."""
    import ctypes
    from .utils.native import rt
    now = now or utcnow()
    nodes = _cstrs([c.node_id for c in acc.contributions])
    seqs = (ctypes.c_longlong * max(len(acc.contributions), 1))(*[c.seq_num for c in acc.contributions])
    weight = ctypes.c_double(0.0)
    reason = ctypes.create_string_buffer(256)
    ok = rt().dts_accept_push(acc.checkpoint_version, push.checkpoint_version, int(max_staleness),
                              len(acc.contributions), nodes, seqs, push.node_id.encode(), push.seq_num,
                              float(push.tokens_processed), float(staleness_decay), ctypes.byref(weight), reason, 256)
    if not ok:
        return False, reason.value.decode()
    acc.contributions = [c for c in acc.contributions if c.node_id != push.node_id]
    acc.contributions.append(ContributionMeta(
        node_id=push.node_id, seq_num=push.seq_num, weight=weight.value, checkpoint_version=push.checkpoint_version,
        inner_steps=push.inner_steps, tokens_processed=push.tokens_processed, delta_key=push.delta_key,
        received_at=now, training_loss=push.training_loss))
    if acc.first_contribution_at is None:
        acc.first_contribution_at = now
    acc.version += 1
    return True, None


def should_checkpoint(acc: AccumulatorState, min_contributions_override: int, cs: CoordinatorPersistentState,
                      now: Optional[_dt.datetime] = None) -> bool:
    """Patience-based trigger (state.rs:140-225), decided by the runtime library's ``dts_should_checkpoint``."""
    import ctypes
    from .utils.native import rt
    if not acc.contributions:
        return False
    now = now or utcnow()
    elapsed = max((now - acc.first_contribution_at).total_seconds(), 0.0) if acc.first_contribution_at else 0.0
    active = list(cs.heartbeats)
    times = []
    for nid in active:
        p = cs.node_profiles.get(nid)
        t = None
        if p is not None:
            t = p.expected_round_time if p.expected_round_time is not None else p.round_time_secs
        times.append(float("nan") if t is None else float(t))
    tarr = (ctypes.c_double * max(len(times), 1))(*times)
    return bool(rt().dts_should_checkpoint(len(acc.contributions), _cstrs([c.node_id for c in acc.contributions]),
                                           len(active), _cstrs(active), tarr, float(elapsed),
                                           int(min_contributions_override)))


def update_round_time(cs: CoordinatorPersistentState, node_id: str, now_secs: Optional[int] = None):
    """Round-time EMA 0.3/0.7 between consecutive pushes in (10, 600) s (routes.rs:244-263), computed by the
    runtime library's ``dts_update_round_time``."""
    from .utils.native import rt
    now_secs = int(time.time()) if now_secs is None else now_secs
    p = cs.node_profiles.get(node_id)
    if p is None:
        return
    prev = float("nan") if p.round_time_secs is None else float(p.round_time_secs)
    last = -1 if p.last_push_time is None else int(p.last_push_time)
    new = rt().dts_update_round_time(prev, last, int(now_secs))
    p.round_time_secs = None if math.isnan(new) else new
    p.last_push_time = now_secs


def clip_scales(norms: List[float]) -> Tuple[List[float], List[float]]:
    """3x running-average norm clip in arrival order (aggregation.rs:310-328).
    Returns (scale per delta, effective norm per delta)."""
    scales, eff = [], []
    for n in norms:
        s, e = 1.0, n
        if eff:
            avg = sum(eff) / len(eff)
            mx = avg * 3.0
            if n > mx and n > 0.0:
                s, e = mx / n, mx
        scales.append(s)
        eff.append(e)
    return scales, eff


def validate_stats(sumsq: float, maxabs: float, nonfinite: bool, empty: bool = False) -> Optional[str]:
    """validate_delta (compression.rs:388-424) from aggregated statistics; None = valid."""
    if empty:
        return "Empty delta"
    if nonfinite:
        return "NaN/Inf in delta"
    if maxabs > 100.0:
        return f"Magnitude too large: {maxabs:.1f}"
    norm = math.sqrt(sumsq)
    if norm > 1000.0:
        return f"Total norm too large: {norm:.1f}"
    if norm < 1e-10:
        return f"Total norm near zero: {norm:.2e}"
    return None


class Accumulator:
    """Coordinator accumulator + trigger with merge single-flight and mid-merge carry-over."""

    def __init__(self, staleness_decay=0.9, max_staleness=10, min_contributions=0, checkpoint_version=0):
        self.state = AccumulatorState(checkpoint_version=checkpoint_version)
        self.cs = CoordinatorPersistentState()
        self.decay, self.max_staleness, self.min_contributions = staleness_decay, max_staleness, min_contributions
        self.merging = False
        self.pending: List[DeltaPush] = []
        self.total_contributions = 0

    def heartbeat(self, node_id: str, now_secs: Optional[int] = None):
        self.cs.heartbeats[node_id] = int(time.time()) if now_secs is None else now_secs
        self.cs.node_profiles.setdefault(node_id, NodeProfile())

    def push(self, p: DeltaPush, now=None):
        if self.merging:
            # arrives during a merge: applied to the next cycle instead of being lost
            self.pending.append(p)
            return True, None
        ok, reason = apply_delta_push(self.state, p, self.decay, self.max_staleness, now)
        if ok:
            update_round_time(self.cs, p.node_id)
        return ok, reason

    def ready(self, now=None) -> bool:
        return not self.merging and should_checkpoint(self.state, self.min_contributions, self.cs, now)

    def begin_merge(self) -> AccumulatorState:
        self.merging = True
        snap = AccumulatorState.from_dict(self.state.to_dict())
        return snap

    def finish_merge(self, new_version: int, contributor_ids: List[str], tokens: int):
        self.state = AccumulatorState(checkpoint_version=new_version, version=self.state.version + 1)
        self.cs.recent_contributors.append((new_version, list(contributor_ids)))
        self.cs.recent_contributors = self.cs.recent_contributors[-5:]
        window = self.cs.recent_contributors[-3:]
        self.cs.active_nodes = len({n for _, ns in window for n in ns})
        self.cs.total_tokens_trained += tokens
        self.total_contributions += len(contributor_ids)
        self.merging = False
        pending, self.pending = self.pending, []
        for p in pending:
            self.push(p)

    def abort_merge(self):
        self.merging = False
        pending, self.pending = self.pending, []
        for p in pending:
            self.push(p)
