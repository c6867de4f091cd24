"""Coordinator: accumulator/trigger state machine (mocked clock) and the HTTP service on localhost
with an FsStore (the reference has no coordinator tests; these restate state.rs / routes.rs /
aggregation.rs behaviour)."""
import datetime as dt
import json
import time

import pytest
import torch

from distrain_b200 import protocol as P
from distrain_b200.config import CoordinatorConfig, CompressionConfig, ModelConfig
from distrain_b200.utils.storage import FsStore
from distrain_b200.utils.checkpoint import load_safetensors_bytes
from distrain_b200.utils.delta_codec import encode_sparse_delta
from distrain_b200.parallel.compression import compress_reference


def _push(node, seq, ver=0, tokens=1000, key=None, loss=5.0):
    return P.DeltaPush(node_id=node, seq_num=seq, checkpoint_version=ver, inner_steps=10,
                       delta_key=key or P.delta_path(ver, node, seq), training_loss=loss, tokens_processed=tokens,
                       training_time_secs=1.0)


def test_apply_delta_push_rules():
    acc = P.AccumulatorState(checkpoint_version=12)
    ok, r = P.apply_delta_push(acc, _push("a", 1, ver=1), 0.9, 10)
    assert not ok and r == "Too stale: 11 > 10"
    ok, _ = P.apply_delta_push(acc, _push("a", 1, ver=10, tokens=100), 0.9, 10)
    assert ok and abs(acc.contributions[0].weight - 100 * 0.81) < 1e-9
    ok, r = P.apply_delta_push(acc, _push("a", 1, ver=10), 0.9, 10)
    assert not ok and r.startswith("Duplicate")
    ok, _ = P.apply_delta_push(acc, _push("a", 2, ver=12, tokens=50), 0.9, 10)
    assert ok and len(acc.contributions) == 1 and acc.contributions[0].seq_num == 2
    assert acc.version == 2 and acc.first_contribution_at is not None


def test_trigger_all_active_min_and_patience():
    cs = P.CoordinatorPersistentState(heartbeats={"a": 1, "b": 1, "c": 1})
    acc = P.AccumulatorState()
    t0 = P.utcnow()
    P.apply_delta_push(acc, _push("a", 1), 0.9, 10, now=t0)
    assert not P.should_checkpoint(acc, 0, cs, now=t0)          # 1 < max(3//2, 2)
    P.apply_delta_push(acc, _push("b", 1), 0.9, 10, now=t0)
    assert not P.should_checkpoint(acc, 0, cs, now=t0 + dt.timedelta(seconds=10))
    assert P.should_checkpoint(acc, 0, cs, now=t0 + dt.timedelta(seconds=61))   # cold-start patience 60 s
    assert P.should_checkpoint(acc, 2, cs, now=t0) is False     # override met, but c missing and patience not over
    P.apply_delta_push(acc, _push("c", 1), 0.9, 10, now=t0)
    assert P.should_checkpoint(acc, 0, cs, now=t0)              # all active contributed
    # patience from profiles: cluster max 1.2x, clamped to [30, 300]
    cs2 = P.CoordinatorPersistentState(heartbeats={"a": 1, "b": 1, "x": 1},
                                       node_profiles={"a": P.NodeProfile(expected_round_time=100.0),
                                                      "b": P.NodeProfile(round_time_secs=110.0),
                                                      "x": P.NodeProfile(expected_round_time=1000.0)})
    acc2 = P.AccumulatorState()
    P.apply_delta_push(acc2, _push("a", 1), 0.9, 10, now=t0)
    P.apply_delta_push(acc2, _push("b", 1), 0.9, 10, now=t0)
    assert not P.should_checkpoint(acc2, 0, cs2, now=t0 + dt.timedelta(seconds=131))
    assert P.should_checkpoint(acc2, 0, cs2, now=t0 + dt.timedelta(seconds=132))


def test_clip_scales_arrival_order():
    s, e = P.clip_scales([1.0, 1.0, 10.0, 2.0])
    assert s[:2] == [1.0, 1.0] and abs(s[2] - 0.3) < 1e-12 and s[3] == 1.0
    assert e == [1.0, 1.0, 3.0, 2.0]


def test_accumulator_carries_over_mid_merge_pushes():
    a = P.Accumulator()
    a.heartbeat("x")
    a.push(_push("x", 1))
    snap = a.begin_merge()
    a.push(_push("y", 1))  # arrives during the merge
    a.finish_merge(1, ["x"], 1000)
    assert [c.node_id for c in a.state.contributions] == ["y"]
    assert a.state.checkpoint_version == 1
    assert a.state.contributions[0].weight == pytest.approx(1000 * 0.9)  # pushed against v0 -> staleness 1


def test_wire_types_roundtrip_reference_shapes():
    js = ('{"node_id":"n1","seq_num":3,"checkpoint_version":2,"inner_steps":5,"delta_key":"k","training_loss":1.5,'
          '"tokens_processed":100,"training_time_secs":2.0}')
    p = P.DeltaPush.from_json(js)
    assert p.compressed_bytes is None and p.tokens_processed == 100
    r = P.DeltaPushResponse(accepted=True, checkpoint_version=4).to_dict()
    assert "reason" not in r
    acc = P.AccumulatorState.from_dict({"checkpoint_version": 1, "contributions": [
        {"node_id": "n", "seq_num": 1, "weight": 2.0, "checkpoint_version": 1, "inner_steps": 3,
         "delta_key": "k", "received_at": "2025-01-02T03:04:05.123456789Z"}], "version": 7})
    assert acc.contributions[0].tokens_processed == 0 and acc.first_contribution_at is None
    assert P.AccumulatorState.from_dict(acc.to_dict()).to_dict() == acc.to_dict()
    assert P.checkpoint_path(3) == "checkpoints/v3/model.safetensors"
    assert P.delta_path(2, "n", 5) == "deltas/v2/n_5.delta.zst"
    assert P.data_shard_path(7) == "data/shard_0007.bin"


@pytest.fixture
def service(tmp_path):
    from distrain_b200.coordinator.service import CoordinatorService, bootstrap
    store = FsStore(str(tmp_path))
    cfg = ModelConfig(hidden_dim=32, num_layers=1, num_heads=2, num_kv_heads=1, ffn_hidden_dim=64, vocab_size=64)
    layout, flat = bootstrap(store, cfg, seed=0)
    ccfg = CoordinatorConfig(min_contributions=0, keep_versions=10)
    svc = CoordinatorService(ccfg, store, flush_interval=3600)
    port = svc.start(host="127.0.0.1", port=0, threads=4)
    yield svc, store, layout, flat, port
    svc.stop()


def test_http_service_end_to_end(service):
    from distrain_b200.coordinator.client import CoordinatorClient
    svc, store, layout, flat, port = service
    cl = CoordinatorClient(f"http://127.0.0.1:{port}")
    assert cl.health()
    reg = cl.register(P.RegisterRequest(gpu_model="B200", gpu_memory_gb=180.0, bandwidth_mbps=1e5, node_id="n1",
                                        hardware={"gpu_model": "B200", "vram_mb": 183359,
                                                  "device_type": "DiscreteGpu", "cpu_cores": 8, "ram_mb": 1000,
                                                  "expected_round_time_secs": 30.0}))
    assert reg.node_id == "n1" and reg.status == "Active" and reg.training_params["lr_max"] == 3e-4
    cl.register(P.RegisterRequest(gpu_model="B200", gpu_memory_gb=180.0, bandwidth_mbps=1e5, node_id="n2"))
    for n in ("n1", "n2"):
        hb = cl.heartbeat(P.HeartbeatRequest(node_id=n, checkpoint_version=0))
    assert hb.active_nodes == 2 and hb.latest_version == 0 and not hb.should_abort
    # two nodes push reference-format deltas through the upload proxy
    sd0 = layout.to_state_dict(flat)
    shapes = {k: list(v.shape) for k, v in sd0.items()}
    for i, n in enumerate(("n1", "n2")):
        torch.manual_seed(i)
        delta = {k: torch.randn(v.numel()) * 1e-3 for k, v in sd0.items()}
        sd, stats = compress_reference(delta, shapes, CompressionConfig(top_k_fraction=0.2), {})
        key = P.delta_path(0, n, 1)
        cl.upload(key, encode_sparse_delta(sd))
        r = cl.push_delta(_push(n, 1, ver=0, key=key, tokens=1000 * (i + 1)))
        assert r.accepted
    for _ in range(200):
        if cl.get_latest_checkpoint().version == 1:
            break
        time.sleep(0.05)
    assert cl.get_latest_checkpoint().version == 1, svc.last_error
    new = load_safetensors_bytes(cl.download(P.checkpoint_path(1)))
    assert set(new) == set(sd0)
    meta = json.loads(cl.download(P.checkpoint_metadata_path(1)))
    assert meta["contributions_accepted"] == 2 and meta["outer_lr"] == 1.0
    hist = [json.loads(l) for l in store.get(P.stats_history_path()).decode().splitlines()]
    assert [h["event"] for h in hist].count("delta_accepted") == 2 and hist[-1]["event"] == "checkpoint_produced"
    st = cl.get_status()
    assert st.checkpoint_version == 1 and st.accumulator_contributions == 0 and st.active_nodes == 2
    m = cl.metrics()
    assert "distrain_checkpoint_version 1" in m and "distrain_delta_pushes_accepted 2" in m
    # after the merge the accumulator starts over: the same (node, seq) is accepted again at staleness 1,
    # a repeat of it is a duplicate, and a push 11 versions behind is too stale
    r = cl.push_delta(_push("n1", 1, ver=0))
    assert r.accepted and r.checkpoint_version == 1
    r = cl.push_delta(_push("n1", 1, ver=0))
    assert not r.accepted and r.reason.startswith("Duplicate")
    svc.acc.state.checkpoint_version = 12
    r = cl.push_delta(_push("n2", 5, ver=1))
    assert not r.accepted and r.reason == "Too stale: 11 > 10"
    svc.acc.state.checkpoint_version = 1
    svc.acc.state.contributions.clear()
    # restart: state reloads from the store
    svc.flush()
    from distrain_b200.coordinator.service import CoordinatorService
    svc2 = CoordinatorService(CoordinatorConfig(), store, flush_interval=3600)
    assert svc2.acc.state.checkpoint_version == 1
    assert svc2.acc.cs.total_tokens_trained == 3000


def test_merge_is_permutation_invariant_without_clipping():
    """The weighted merge is commutative (paper p.3 sec 3.1): with deltas of similar norm (no 3x clip fires)
    any arrival order gives the same checkpoint within fp32 rounding. The clip itself uses the running
    average in arrival order, as in the reference, so an outlier's scale can depend on the order."""
    import itertools
    from distrain_b200.parallel.merge import merge_reference
    g = torch.Generator().manual_seed(0)
    ck = {"a": torch.randn(300, generator=g), "b": torch.randn(7, 5, generator=g)}
    deltas = [{k: torch.randn(v.shape, generator=g) * 1e-3 * (1 + 0.1 * i) for k, v in ck.items()} for i in range(4)]
    weights = [1000.0, 750.0 * 0.9, 500.0 * 0.81, 2000.0]
    base, _, _ = merge_reference(ck, deltas, weights)
    for perm in itertools.permutations(range(4)):
        got, _, info = merge_reference(ck, [deltas[i] for i in perm], [weights[i] for i in perm])
        assert info["accepted"] == 4
        for k in ck:
            torch.testing.assert_close(got[k], base[k], rtol=1e-6, atol=1e-7)


def test_nesterov_outer_step_golden_numbers():
    """Outer Nesterov step with lr 0.7, momentum 0.9 from zero velocity: v = avg, theta -= lr * (mu * v + avg)
    (the reference's worked example, core/model/src/training.rs:347-365), then a second step."""
    import torch
    from distrain_b200.parallel.merge import nesterov_step
    ck = {"w": torch.tensor([1.0, 2.0, 3.0], dtype=torch.float64)}
    avg = {"w": torch.tensor([0.1, 0.2, 0.3], dtype=torch.float64)}
    ck, vel = nesterov_step(ck, avg, None, 0.7, 0.9)
    assert torch.allclose(vel["w"], avg["w"])
    assert torch.allclose(ck["w"], torch.tensor([0.867, 1.734, 2.601], dtype=torch.float64), atol=1e-12)
    ck, vel = nesterov_step(ck, avg, vel, 0.7, 0.9)
    assert torch.allclose(vel["w"], torch.tensor([0.19, 0.38, 0.57], dtype=torch.float64), atol=1e-12)
    assert torch.allclose(ck["w"], torch.tensor([0.867 - 0.7 * 0.271, 1.734 - 0.7 * 0.542, 2.601 - 0.7 * 0.813],
                                                dtype=torch.float64), atol=1e-12)


def test_http_body_limits(service):
    """The reference's 512 MB request-body cap (coordinator/src/main.rs:128): a larger Content-Length is
    refused with 413 before any body is read; chunked uploads are refused with 411 (Content-Length only)."""
    import socket
    _, _, _, _, port = service

    def raw(req: bytes) -> bytes:
        with socket.create_connection(("127.0.0.1", port), timeout=10) as s:
            s.sendall(req)
            return s.recv(4096)
    r = raw(b"PUT /upload/deltas/v0/x.delta.zst HTTP/1.1\r\nHost: c\r\nContent-Length: %d\r\n\r\n" % (600 << 20))
    assert r.split(b"\r\n")[0].split()[1] == b"413"
    r = raw(b"PUT /upload/deltas/v0/x.delta.zst HTTP/1.1\r\nHost: c\r\nTransfer-Encoding: chunked\r\n\r\n5\r\nhello\r\n0\r\n\r\n")
    assert r.split(b"\r\n")[0].split()[1] == b"411"
    r = raw(b"GET /health HTTP/1.1\r\nHost: c\r\nContent-Length: 0\r\n\r\n")  # the server keeps serving
    assert r.split(b"\r\n")[0].split()[1] == b"200"
    # permissive CORS with preflight, for browser nodes (the reference's CorsLayer::permissive)
    r = raw(b"OPTIONS /delta HTTP/1.1\r\nHost: c\r\nOrigin: http://x\r\nAccess-Control-Request-Method: POST\r\n\r\n")
    assert r.split(b"\r\n")[0].split()[1] in (b"200", b"204") and b"Access-Control-Allow-Origin: *" in r


def test_config_route_secret_can_be_withheld(service):
    """GET /config gives nodes the storage credentials (the reference's behaviour); with
    PUBLISH_STORAGE_SECRET=0 the secret is withheld and the rest of the reply is unchanged."""
    from distrain_b200.config import CoordinatorConfig
    from distrain_b200.coordinator.client import CoordinatorClient
    svc, _, _, _, port = service
    cl = CoordinatorClient(f"http://127.0.0.1:{port}")
    full = cl.get_config()
    assert full["storage"]["secret_access_key"] == svc.cfg.storage.secret_access_key != ""
    svc.cfg.publish_storage_secret = CoordinatorConfig.from_env({"PUBLISH_STORAGE_SECRET": "0"}).publish_storage_secret
    red = cl.get_config()
    assert red["storage"]["secret_access_key"] == ""
    assert {k: v for k, v in red["storage"].items() if k != "secret_access_key"} == \
        {k: v for k, v in full["storage"].items() if k != "secret_access_key"}
    assert CoordinatorConfig.from_env({}).publish_storage_secret is True


def test_outer_lr_before_and_after_a_reported_loss(tmp_path):
    """The merged delta is applied unscaled once contributions report a training loss; with no loss reported
    the configured initial outer lr applies. state/outer_lr.json keeps the applied lr and the last norms."""
    import time as _time
    from distrain_b200.config import CompressionConfig, CoordinatorConfig, ModelConfig
    from distrain_b200.coordinator.client import CoordinatorClient
    from distrain_b200.coordinator.service import CoordinatorService, bootstrap
    from distrain_b200.parallel.compression import compress_reference
    from distrain_b200.utils.checkpoint import load_safetensors_bytes
    from distrain_b200.utils.delta_codec import decode_delta, encode_sparse_delta
    import torch
    store = FsStore(str(tmp_path))
    cfg = ModelConfig(hidden_dim=32, num_layers=1, num_heads=2, num_kv_heads=1, ffn_hidden_dim=64, vocab_size=64)
    layout, flat = bootstrap(store, cfg, seed=0)
    svc = CoordinatorService(CoordinatorConfig(min_contributions=0, outer_lr=0.25), store, flush_interval=3600)
    port = svc.start(host="127.0.0.1", port=0, threads=4)
    cl = CoordinatorClient(f"http://127.0.0.1:{port}")
    try:
        cl.register(P.RegisterRequest(gpu_model="cpu", gpu_memory_gb=0.0, bandwidth_mbps=0.0, node_id="n"))
        cl.heartbeat(P.HeartbeatRequest(node_id="n", checkpoint_version=0))  # the one active node
        for v, loss, want_lr in ((0, 0.0, 0.25), (1, 3.5, 1.0)):
            ck = load_safetensors_bytes(store.get(P.checkpoint_path(v)))
            g = torch.Generator().manual_seed(v)
            delta = {k: torch.randn(t.numel(), generator=g) * 1e-3 for k, t in ck.items()}
            sd, _ = compress_reference(delta, {k: list(t.shape) for k, t in ck.items()},
                                       CompressionConfig(top_k_fraction=0.3), {})
            blob = encode_sparse_delta(sd)
            cl.upload(P.delta_path(v, "n", v + 1), blob)
            assert cl.push_delta(P.DeltaPush(node_id="n", seq_num=v + 1, checkpoint_version=v, inner_steps=10,
                                             delta_key=P.delta_path(v, "n", v + 1), training_loss=loss,
                                             tokens_processed=100, training_time_secs=1.0)).accepted
            t0 = _time.time()
            while cl.get_latest_checkpoint().version < v + 1 and _time.time() - t0 < 30:
                _time.sleep(0.05)
            new = load_safetensors_bytes(store.get(P.checkpoint_path(v + 1)))
            dec = decode_delta(blob)
            for k in ck:
                assert torch.allclose(new[k].reshape(-1), ck[k].reshape(-1) - want_lr * dec[k].reshape(-1), atol=1e-7)
            st = store.get_json(P.outer_lr_state_path())
            assert st["outer_lr"] == want_lr and st["outer_momentum"] == 0.0 and len(st["recent_norms"]) == v + 1
            assert json.loads(store.get(P.checkpoint_metadata_path(v + 1)))["outer_lr"] == want_lr
    finally:
        svc.stop()
