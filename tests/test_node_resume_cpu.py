"""Node-local resume file of an HTTP node (CPU backend): a node stopped after a round boundary and
restarted on the same checkpoint continues exactly (its next losses equal the ones the stopped node
computed for the same steps: weights, AdamW moments and the data position were restored); restarted
after the coordinator merged a newer checkpoint, it keeps its identity, sequence numbers, step count and
data position and takes the new checkpoint."""
import os
import time

import pytest
import torch

from distrain_b200.config import CompressionConfig, CoordinatorConfig, ModelConfig, OptimConfig
from distrain_b200.coordinator.client import CoordinatorClient
from distrain_b200.coordinator.service import CoordinatorService, bootstrap
from distrain_b200.parallel.http_node import HttpNode
from distrain_b200.utils.data import ShardLoader, SyntheticTokens, prepare_random_shards
from distrain_b200.utils.storage import FsStore

CFG = ModelConfig(hidden_dim=32, num_layers=1, num_heads=2, num_kv_heads=1, ffn_hidden_dim=64, vocab_size=64,
                  max_seq_len=32, rope_theta=10000.0)


def _service(tmp_path, min_contributions):
    store = FsStore(str(tmp_path / "store"))
    bootstrap(store, CFG, seed=0)
    svc = CoordinatorService(CoordinatorConfig(min_contributions=min_contributions, outer_lr=1.0, outer_momentum=0.0),
                             store, flush_interval=3600)
    port = svc.start(host="127.0.0.1", port=0, threads=4)
    return store, svc, f"http://127.0.0.1:{port}"


def _node(url, store, data, resume, node_id=None):
    return HttpNode(url, store, CFG, batch=2, seq_len=17, h_mini=5, optim=OptimConfig(lr=3e-3),
                    compression=CompressionConfig(top_k_fraction=0.2), device="cpu", node_id=node_id, data=data,
                    poll_secs=0.1, resume_path=resume)


@pytest.mark.timeout(300)
def test_restart_on_the_same_checkpoint_continues_exactly(tmp_path):
    # more contributions required than there are nodes: no merge, the checkpoint stays at v0
    store, svc, url = _service(tmp_path, min_contributions=10)
    shards = tmp_path / "data"
    prepare_random_shards(str(shards), 2, 20_000, CFG.vocab_size, seed=5)
    paths = [str(shards / f"shard_{i:04d}.bin") for i in range(2)]
    resume = str(tmp_path / "node.resume")
    try:
        a = _node(url, store, ShardLoader(paths, 17, 2).next_batch, resume)
        a.register()
        log_a = a.run(12)  # pushes after steps 5 and 10; the file holds the boundary after step 10
        assert not a.errors and [p["seq"] for p in a.pushes] == [1, 2]
        rec = torch.load(resume, weights_only=False)
        assert (rec["seq"], rec["global_step"], rec["version"], rec["node_id"]) == (2, 10, 0, a.node_id)
        assert rec["ef"] and rec["optimizer"]["t"] == 10
        b = _node(url, store, ShardLoader(paths, 17, 2).next_batch, resume)
        assert b.node_id == a.node_id  # identity from the file, before registering
        b.register()
        log_b = b.run(16)
        assert b.resumed == "exact" and not b.errors
        assert [x["step"] for x in log_b] == [11, 12, 13, 14, 15, 16]
        # steps 11 and 12 repeat exactly what the stopped node computed from the same state and batches
        assert [x["loss"] for x in log_b[:2]] == pytest.approx([x["loss"] for x in log_a[10:12]], rel=1e-6)
        assert [p["seq"] for p in b.pushes] == [3]  # sequence numbers continue
    finally:
        svc.stop()


@pytest.mark.timeout(300)
def test_restart_after_a_newer_checkpoint_keeps_identity_and_position(tmp_path):
    store, svc, url = _service(tmp_path, min_contributions=0)  # a single node's push is merged at once
    resume = str(tmp_path / "node.resume")
    try:
        src_a = SyntheticTokens(CFG.vocab_size, 2, 17, seed=9)
        a = _node(url, store, src_a.next_batch, resume, node_id="node-r")
        a.register()
        a.run(11)
        assert not a.errors
        cl = CoordinatorClient(url)
        t0 = time.time()
        while cl.get_latest_checkpoint().version < 1 and time.time() - t0 < 60:  # the merge is asynchronous
            time.sleep(0.1)
        latest = cl.get_latest_checkpoint().version
        rec = torch.load(resume, weights_only=False)
        assert latest > rec["version"] == 0
        src_b = SyntheticTokens(CFG.vocab_size, 2, 17, seed=12345)  # restored from the file, not this seed
        b = _node(url, store, src_b.next_batch, resume)
        b.register()
        assert b.node_id == "node-r"
        want_next = SyntheticTokens(CFG.vocab_size, 2, 17, seed=9)
        want_next.restore(rec["data"])
        b.run(rec["global_step"] + 1)  # one more step
        assert b.resumed == "identity" and b.version == latest and not b.errors
        assert b.log[0]["step"] == rec["global_step"] + 1
        want_next.next_batch()  # the one batch that step consumed
        assert torch.equal(src_b.g.get_state(), want_next.g.get_state())
    finally:
        svc.stop()


def test_loader_seek_roundtrip(tmp_path):
    prepare_random_shards(str(tmp_path), 3, 5_000, 64, seed=1)
    paths = [str(tmp_path / f"shard_{i:04d}.bin") for i in range(3)]
    a = ShardLoader(paths, 16, 4)
    for _ in range(90):  # crosses into the second shard
        a.next_batch()
    st = a.state()
    assert st["shard"] == 1
    want = a.next_batch()
    b = ShardLoader(paths, 16, 4)
    b.restore(st)
    assert torch.equal(b.next_batch(), want)
    with pytest.raises(Exception):
        b.restore({"shard": 7, "offset": 0})
    assert os.path.exists(paths[0])


@pytest.mark.timeout(300)
def test_node_stops_under_host_memory_pressure(tmp_path, monkeypatch):
    from distrain_b200.parallel import http_node
    store, svc, url = _service(tmp_path, min_contributions=10)
    try:
        monkeypatch.setattr(http_node, "memory_pressure", lambda frac: True)
        n = _node(url, store, SyntheticTokens(CFG.vocab_size, 2, 17, seed=1).next_batch, None)
        n.register()
        log = n.run(50)
        assert len(log) == 10 and any("host memory pressure" in e for e in n.errors)  # checked every 10 steps
    finally:
        svc.stop()


@pytest.mark.timeout(300)
def test_start_streams_the_nodes_assigned_shards_from_the_store(tmp_path, capsys):
    """`start` without --data-dir reads the shards that the deterministic assignment gives this node id
    from the store's data/ prefix (fetched into its cache), like the reference node."""
    import json
    from distrain_b200 import cli
    from distrain_b200.config import TrainingParams
    from distrain_b200.utils.native import shard_assignment
    store, svc, url = _service(tmp_path, min_contributions=10)
    try:
        cli.main(["prepare-data", "--output-dir", str(tmp_path / "prep"), "--num-shards", "10",
                  "--tokens-per-shard", "5000", "--vocab", str(CFG.vocab_size), "--upload-store",
                  str(tmp_path / "store")])
        cache = tmp_path / "cache"
        cli.main(["start", "--coordinator-url", url, "--store", str(tmp_path / "store"), "--cpu", "--steps", "6",
                  "--batch-size", "2", "--seq-len", "17", "--h-mini", "5", "--node-id", "streamer",
                  "--cache-dir", str(cache), "--poll-secs", "0.2"])
        out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
        assert out["event"] == "node_done" and out["steps"] == 6 and not out["errors"]
        want = shard_assignment("streamer", 0, 10, TrainingParams().shards_per_node(10))
        assert sorted(f for f in os.listdir(cache) if f.endswith(".bin")) == sorted(f"shard_{i:04d}.bin" for i in want)
        # a restart without --node-id takes the identity kept in the cache directory
        cli.main(["start", "--coordinator-url", url, "--store", str(tmp_path / "store"), "--cpu", "--steps", "3",
                  "--batch-size", "2", "--seq-len", "17", "--h-mini", "5", "--cache-dir", str(cache),
                  "--poll-secs", "0.2"])
        assert json.loads(capsys.readouterr().out.strip().splitlines()[-1])["node_id"] == "streamer"
    finally:
        svc.stop()


@pytest.mark.timeout(300)
def test_push_interval_follows_the_bandwidth_recommendation(tmp_path):
    """With (min, max) inner-step bounds the push interval is retuned at each checkpoint swap from the
    upload rate (steps that upload in ~10 s); local uploads are fast, so it rises to the maximum."""
    store, svc, url = _service(tmp_path, min_contributions=0)
    try:
        n = _node(url, store, SyntheticTokens(CFG.vocab_size, 2, 17, seed=3).next_batch, None, node_id="tuned")
        n.h_mini_bounds = (5, 8)
        n.register()
        n.run(150)  # CPU steps are far faster than a merge round trip: leave room for swaps and 8-step rounds
        assert not n.errors and n.version >= 1
        assert n.recommended_h_mini >= 8 and n.h_mini == 8
        assert any(e["inner_steps"] == 8 for e in _accepted(store, "tuned"))  # rounds of 8 steps after a swap
    finally:
        svc.stop()


def _accepted(store, node_id):
    import json
    from distrain_b200 import protocol as P
    raw = store.get(P.stats_history_path()).decode()
    return [e for e in map(json.loads, raw.splitlines()) if e["event"] == "delta_accepted" and e["node_id"] == node_id]


@pytest.mark.timeout(300)
def test_checkpoint_cache_keeps_the_newest_three(tmp_path):
    """Checkpoints fetched from the store are cached on disk (newest 3 kept): a restarted node reads an
    unchanged checkpoint from its cache instead of the store."""
    store, svc, url = _service(tmp_path, min_contributions=0)
    cache = tmp_path / "cache"
    try:
        n = _node(url, store, SyntheticTokens(CFG.vocab_size, 2, 17, seed=4).next_batch, None, node_id="cached")
        n.ckpt_cache_dir = str(cache)
        n.register()
        n.run(150)
        assert not n.errors and n.version >= 3  # v0..v3 fetched: four checkpoints, three kept
        # the checkpoint thread may have fetched versions newer than the one the node last swapped to
        kept = sorted(os.listdir(cache / "checkpoints"), key=lambda f: int(f[1:].split(".")[0]))
        newest = int(kept[-1][1:].split(".")[0])
        assert len(kept) == 3 and newest >= n.version
        gets = []
        real_get = store.get
        store.get = lambda key: (gets.append(key), real_get(key))[1]
        m = _node(url, store, SyntheticTokens(CFG.vocab_size, 2, 17, seed=5).next_batch, None, node_id="cached")
        m.ckpt_cache_dir = str(cache)
        assert m._load_version(newest) is not None
        assert not any(k.startswith("checkpoints/") for k in gets)
    finally:
        svc.stop()


def test_loss_spike_skips_the_update_on_the_cpu_backend():
    """A step whose loss exceeds the spike bound leaves weights and optimizer untouched."""
    from distrain_b200.config import OptimConfig
    from distrain_b200.models.params import ParamLayout, init_flat
    from distrain_b200.parallel.http_node import CpuBackend
    b = CpuBackend(CFG, OptimConfig(lr=1e-2))
    L = ParamLayout(CFG)
    b.load(L.to_state_dict(init_flat(L, 0.02, 0)))
    toks = SyntheticTokens(CFG.vocab_size, 2, 17, seed=2).next_batch()
    before = b.state()
    loss = b.step(toks, 1e-2, max_loss=0.1)  # any real loss is a "spike" against this bound
    assert loss > 0.1 and b.opt.t == 0
    assert all(torch.equal(before[k], v) for k, v in b.state().items())
    b.step(toks, 1e-2, max_loss=None)
    assert b.opt.t == 1 and not all(torch.equal(before[k], v) for k, v in b.state().items())
