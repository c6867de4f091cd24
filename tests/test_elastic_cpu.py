"""Elastic membership over HTTP with real node processes (CPU, micro model): three nodes train against
the coordinator; one node process is killed mid-run; the others keep merging (the dead node still
counts as active until its heartbeat expires, so a merge waits for the patience window, at least 30 s,
and then goes ahead without it); a fourth node that joins later has its pushes accepted and merged."""
import json
import os
import subprocess
import sys
import time

from distrain_b200 import protocol as P
from distrain_b200.config import CoordinatorConfig, ModelConfig
from distrain_b200.coordinator.client import CoordinatorClient
from distrain_b200.coordinator.service import CoordinatorService, bootstrap
from distrain_b200.utils.storage import FsStore

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _events(store):
    try:
        raw = store.get(P.stats_history_path()).decode()
    except Exception:
        return []
    return [json.loads(line) for line in raw.splitlines() if line.strip()]


def _wait(pred, secs, what):
    t0 = time.time()
    while time.time() - t0 < secs:
        if pred():
            return
        time.sleep(0.25)
    raise AssertionError(f"timed out after {secs} s waiting for {what}")


def test_killed_node_does_not_block_merges_and_a_late_node_joins(tmp_path):
    store = FsStore(str(tmp_path))
    cfg = ModelConfig(hidden_dim=32, num_layers=1, num_heads=2, num_kv_heads=1, ffn_hidden_dim=64, vocab_size=64)
    bootstrap(store, cfg, seed=0)
    svc = CoordinatorService(CoordinatorConfig(min_contributions=0, outer_lr=1.0, outer_momentum=0.0), store,
                             flush_interval=3600)
    port = svc.start(host="127.0.0.1", port=0, threads=4)
    url = f"http://127.0.0.1:{port}"
    cl = CoordinatorClient(url)
    env = dict(os.environ, PYTHONPATH=ROOT, DT_LOG="warning", OMP_NUM_THREADS="1", MKL_NUM_THREADS="1")
    procs = {}

    def start(i):
        procs[i] = subprocess.Popen([sys.executable, "-m", "distrain_b200", "start", "--coordinator-url", url,
                                     "--store", str(tmp_path), "--cpu", "--steps", "1000000", "--batch-size", "2",
                                     "--seq-len", "16", "--h-mini", "10", "--node-id", f"n{i}", "--seed", str(i),
                                     "--poll-secs", "0.5"], env=env, stdout=subprocess.DEVNULL,
                                    stderr=subprocess.DEVNULL)
    try:
        for i in range(3):
            start(i)
        _wait(lambda: {e.get("node_id") for e in _events(store) if e["event"] == "delta_accepted"} >= {"n0", "n1", "n2"},
              180, "an accepted push from every node")
        _wait(lambda: cl.get_latest_checkpoint().version >= 1, 180, "the first merge")
        procs[2].kill()  # the process we started, by its own handle
        procs[2].wait(timeout=30)
        t_kill, ts_kill = time.time(), P.to_rfc3339(P.utcnow())
        v_kill = cl.get_latest_checkpoint().version
        start(3)
        _wait(lambda: any(e["event"] == "delta_accepted" and e["node_id"] == "n3" for e in _events(store)), 180,
              "the late node's first accepted push")
        joined_at = len(_events(store))
        # the dead node still counts as active (heartbeat TTL 10 min), so this merge waits for the patience
        # window and then goes ahead with the nodes that pushed
        _wait(lambda: any(e["event"] == "checkpoint_produced" and e["contributions"] >= 3
                          for e in _events(store)[joined_at:]), 240, "a merge with the late node")
        assert cl.get_latest_checkpoint().version > v_kill
        assert time.time() - t_kill >= 25  # the silent node was waited for (patience >= 30 s), not ignored
        assert all(procs[i].poll() is None for i in (0, 1, 3))  # the other nodes kept running
        assert not any(e["event"] == "delta_accepted" and e["node_id"] == "n2" and e["timestamp"] > ts_kill
                       for e in _events(store))
    finally:
        for p in procs.values():
            if p.poll() is None:
                p.kill()
                p.wait(timeout=30)
        svc.stop()
