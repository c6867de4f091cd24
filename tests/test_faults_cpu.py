"""Host-side fault injection against the coordinator service and its protocol (no GPU involved):

* a corrupt delta and a NaN-poisoned delta are rejected while the merge goes on with the valid one;
* an object-store write failure fails one merge attempt, which is retried with the same contributions
  once the store recovers;
* a node that stops heartbeating stops counting as active after the 10-minute TTL, so the others merge
  without it; a node that heartbeats but never pushes delays the merge by the patience window only;
* a push lost in transit is covered by the node's next sequence number, and the late copy is a duplicate;
* a coordinator restart keeps the contributions waiting in the accumulator.
"""
import datetime as dt
import json
import time

import torch

from distrain_b200 import protocol as P
from distrain_b200.config import CompressionConfig, CoordinatorConfig, ModelConfig
from distrain_b200.coordinator.client import CoordinatorClient
from distrain_b200.coordinator.service import CoordinatorService, bootstrap
from distrain_b200.parallel.compression import compress_reference
from distrain_b200.utils.delta_codec import encode_dtz, encode_sparse_delta
from distrain_b200.utils.storage import FsStore, StorageError


class FaultyStore(FsStore):
    """An FsStore whose next `fail` writes under `prefix` raise."""

    def __init__(self, root):
        super().__init__(root)
        self.prefix, self.fail = None, 0

    def put(self, key, data):
        if self.prefix is not None and self.fail > 0 and key.startswith(self.prefix):
            self.fail -= 1
            raise StorageError(f"injected write failure: {key}")
        return super().put(key, data)


def _cfg():
    return ModelConfig(hidden_dim=32, num_layers=1, num_heads=2, num_kv_heads=1, ffn_hidden_dim=64, vocab_size=64)


def _start(store, **kw):
    svc = CoordinatorService(CoordinatorConfig(min_contributions=0, keep_versions=10, **kw), store,
                             flush_interval=3600)
    port = svc.start(host="127.0.0.1", port=0, threads=4)
    return svc, CoordinatorClient(f"http://127.0.0.1:{port}")


def _join(cl, *nodes):
    for n in nodes:
        cl.register(P.RegisterRequest(gpu_model="cpu", gpu_memory_gb=0.0, bandwidth_mbps=0.0, node_id=n))
        cl.heartbeat(P.HeartbeatRequest(node_id=n, checkpoint_version=0))


def _valid_delta(layout, flat, seed):
    sd0 = layout.to_state_dict(flat)
    shapes = {k: list(v.shape) for k, v in sd0.items()}
    g = torch.Generator().manual_seed(seed)
    delta = {k: torch.randn(v.numel(), generator=g) * 1e-3 for k, v in sd0.items()}
    sd, _ = compress_reference(delta, shapes, CompressionConfig(top_k_fraction=0.2), {})
    return encode_sparse_delta(sd)


def _push(cl, node, seq, key, ver=0, tokens=1000):
    return cl.push_delta(P.DeltaPush(node_id=node, seq_num=seq, checkpoint_version=ver, inner_steps=10,
                                     delta_key=key, training_loss=4.0, tokens_processed=tokens,
                                     training_time_secs=1.0))


def _wait_version(cl, v, secs=20.0):
    t0 = time.time()
    while time.time() - t0 < secs:
        if cl.get_latest_checkpoint().version >= v:
            return True
        time.sleep(0.05)
    return False


def test_corrupt_and_nan_deltas_are_rejected_and_the_merge_goes_on(tmp_path):
    store = FsStore(str(tmp_path))
    layout, flat = bootstrap(store, _cfg(), seed=0)
    svc, cl = _start(store)
    try:
        _join(cl, "good", "corrupt", "poisoned")
        cl.upload(P.delta_path(0, "good", 1), _valid_delta(layout, flat, 1))
        cl.upload(P.delta_path(0, "corrupt", 1), b"\x00\x01 not a delta \xff" * 7)
        n = layout.num_params()
        vals = torch.full((8,), 1e-3)
        vals[3] = float("nan")
        cl.upload(P.delta_path(0, "poisoned", 1), encode_dtz(n, torch.arange(8, dtype=torch.int32), None, None, vals, 0))
        for node in ("good", "corrupt", "poisoned"):
            assert _push(cl, node, 1, P.delta_path(0, node, 1)).accepted  # bytes are only read by the merge
        assert _wait_version(cl, 1), svc.last_error
        meta = json.loads(cl.download(P.checkpoint_metadata_path(1)))
        assert meta["contributions_accepted"] == 1 and meta["contributions_rejected"] == 2
    finally:
        svc.stop()


def test_store_write_failure_fails_one_attempt_then_the_merge_is_retried(tmp_path):
    store = FaultyStore(str(tmp_path))
    layout, flat = bootstrap(store, _cfg(), seed=0)
    store.prefix, store.fail = "checkpoints/v1/", 1
    svc, cl = _start(store)
    try:
        _join(cl, "a", "b")
        for i, node in enumerate(("a", "b")):
            cl.upload(P.delta_path(0, node, 1), _valid_delta(layout, flat, 10 + i))
            assert _push(cl, node, 1, P.delta_path(0, node, 1)).accepted
        assert _wait_version(cl, 1), svc.last_error
        assert svc.metrics.aggregations_failed >= 1 and store.fail == 0
        meta = json.loads(cl.download(P.checkpoint_metadata_path(1)))
        assert meta["contributions_accepted"] == 2  # the retry merged the same two contributions
    finally:
        svc.stop()


def test_dead_node_expires_and_the_others_merge(tmp_path):
    store = FsStore(str(tmp_path))
    layout, flat = bootstrap(store, _cfg(), seed=0)
    svc, cl = _start(store)
    try:
        _join(cl, "alive", "dead")
        # "dead" stopped heartbeating 11 minutes ago; the next heartbeat of anyone prunes it (10 min TTL)
        with svc.lock:
            svc.acc.cs.heartbeats["dead"] = int(time.time()) - 11 * 60
        cl.heartbeat(P.HeartbeatRequest(node_id="alive", checkpoint_version=0))
        assert set(svc.acc.cs.heartbeats) == {"alive"}
        cl.upload(P.delta_path(0, "alive", 1), _valid_delta(layout, flat, 3))
        assert _push(cl, "alive", 1, P.delta_path(0, "alive", 1)).accepted
        assert _wait_version(cl, 1), svc.last_error  # one active node: its contribution suffices
    finally:
        svc.stop()


def test_silent_node_delays_the_merge_by_the_patience_window_only():
    acc = P.Accumulator(min_contributions=0)
    for n in ("a", "b", "c"):
        acc.heartbeat(n)
    t0 = dt.datetime(2026, 1, 1, tzinfo=dt.timezone.utc)
    for n in ("a", "b"):
        ok, _ = acc.push(P.DeltaPush(node_id=n, seq_num=1, checkpoint_version=0, inner_steps=10, delta_key="k",
                                     training_loss=1.0, tokens_processed=100, training_time_secs=1.0), now=t0)
        assert ok
    acc.state.first_contribution_at = t0
    assert not acc.ready(now=t0 + dt.timedelta(seconds=59))  # "c" silent, no round timings: 60 s patience
    assert acc.ready(now=t0 + dt.timedelta(seconds=60))


def test_lost_push_is_covered_by_the_next_sequence_number(tmp_path):
    store = FsStore(str(tmp_path))
    bootstrap(store, _cfg(), seed=0)
    svc, cl = _start(store)
    try:
        _join(cl, "n", "other")
        # seq 1 never arrives; seq 2 does; the late copy of seq 1 is then a duplicate
        assert _push(cl, "n", 2, "deltas/v0/n_2.delta.zst").accepted
        r = _push(cl, "n", 1, "deltas/v0/n_1.delta.zst")
        assert not r.accepted and r.reason == "Duplicate: existing seq_num 2 >= 1"
    finally:
        svc.stop()


def test_restart_keeps_waiting_contributions(tmp_path):
    store = FsStore(str(tmp_path))
    layout, flat = bootstrap(store, _cfg(), seed=0)
    svc, cl = _start(store)
    _join(cl, "a", "b")
    cl.upload(P.delta_path(0, "a", 1), _valid_delta(layout, flat, 7))
    assert _push(cl, "a", 1, P.delta_path(0, "a", 1)).accepted
    assert cl.get_latest_checkpoint().version == 0  # two active nodes: waits for "b"
    svc.flush()
    svc.stop()
    svc2, cl2 = _start(store)
    try:
        assert [c.node_id for c in svc2.acc.state.contributions] == ["a"]
        with svc2.lock:  # the restarted coordinator has seen both nodes recently
            now = int(time.time())
            svc2.acc.cs.heartbeats.update({"a": now, "b": now})
        cl2.upload(P.delta_path(0, "b", 1), _valid_delta(layout, flat, 8))
        assert _push(cl2, "b", 1, P.delta_path(0, "b", 1)).accepted
        assert _wait_version(cl2, 1), svc2.last_error
        meta = json.loads(cl2.download(P.checkpoint_metadata_path(1)))
        assert meta["contributions_accepted"] == 2
    finally:
        svc2.stop()
