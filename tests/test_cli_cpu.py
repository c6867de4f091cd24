"""CLI end to end on CPU: bootstrap, coordinator + two node processes on the micro-test workload,
eval / baseline / generate / status / prepare-data."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PY = [sys.executable, "-m", "distrain_b200"]


def run(args, **kw):
    return subprocess.run(PY + args, cwd=ROOT, capture_output=True, text=True, timeout=600, **kw)


@pytest.mark.timeout(900)
def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_micro_cluster_processes(tmp_path):
    r = run(["micro-cluster", "--nodes", "2", "--steps", "45", "--port", str(_free_port()), "--store",
             str(tmp_path / "s")])
    assert r.returncode == 0, r.stderr[-3000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    for n in out["nodes"]:
        assert n["steps"] == 45 and n["accepted"] >= 1 and not n["errors"], n
        # uniform-random tokens: the loss sits at the entropy floor ln(32768) = 10.397 (no signal to learn)
        assert abs(n["last_loss"] - 10.397) < 0.3, n
    # a node that finishes its steps before the first merge is published exits at version 0; the merge
    # itself must have happened (at least one node swapped, and v1 is in the store)
    assert max(n["version"] for n in out["nodes"]) >= 1, out["nodes"]
    assert os.path.exists(tmp_path / "s" / "distrain-training" / "checkpoints" / "v1" / "model.safetensors")


def test_bootstrap_eval_baseline_generate(tmp_path):
    st = str(tmp_path / "store")
    r = run(["bootstrap", "--preset", "micro", "--store", st])
    assert r.returncode == 0, r.stderr
    ck = os.path.join(st, "distrain-training", "checkpoints", "v0", "model.safetensors")
    r = run(["eval", ck, "--batches", "2", "--batch-size", "2", "--seq-len", "17", "--device", "cpu"])
    assert r.returncode == 0, r.stderr
    loss = json.loads(r.stdout)[0]["loss"]
    assert abs(loss - 5.545) < 0.5  # ~ln(256) at init
    out = str(tmp_path / "b.jsonl")
    r = run(["baseline", ck, "--cpu", "--steps", "10", "--batch-size", "2", "--seq-len", "17", "--output", out])
    assert r.returncode == 0, r.stderr
    rows = [json.loads(l) for l in open(out)]
    # 20% linear warm-up (2 steps) then cosine decay to 0.1 x lr_max
    assert len(rows) == 10 and rows[0]["lr"] == 0.0 and rows[2]["lr"] == pytest.approx(3e-4)
    assert rows[-1]["tokens"] == 10 * 2 * 17 and rows[-1]["lr"] < rows[2]["lr"]
    r = run(["generate", ck, "--prompt-ids", "1,2,3", "--max-tokens", "5"])
    assert r.returncode == 0, r.stderr
    assert len(json.loads(r.stdout)["ids"]) == 8
    r = run(["prepare-data", "--output-dir", str(tmp_path / "d"), "--num-shards", "2", "--tokens-per-shard", "1000",
             "--vocab", "256"])
    assert r.returncode == 0 and json.loads(r.stdout)["total_tokens"] == 2000
    r = run(["eval", ck, "--batches", "1", "--batch-size", "2", "--seq-len", "17", "--data-dir", str(tmp_path / "d"),
             "--device", "cpu"])
    assert r.returncode == 0, r.stderr


def test_batch_calibration_binary_search(monkeypatch):
    """Unset batch size on a GPU node: probes in child processes, binary search for the largest that fits."""
    import subprocess as sp
    from distrain_b200 import cli
    probes = []

    def fake_run(cmd, **kw):
        b = int(cmd[cmd.index("--batch-size") + 1])
        probes.append(b)
        return sp.CompletedProcess(cmd, 0 if b <= 37 else 3)
    monkeypatch.setattr(cli.subprocess, "run", fake_run)
    assert cli.calibrate_batch_size("ck.safetensors", 512, device="cuda:0") == 37
    assert len(probes) <= 9 and probes[0] == 128
    probes.clear()
    monkeypatch.setattr(cli.subprocess, "run", lambda cmd, **kw: sp.CompletedProcess(cmd, 3))
    with pytest.raises(SystemExit):
        cli._calibrated_batch(b"not used by the fake probe", 512, "cuda:0")


def test_oom_halves_the_batch_under_the_same_identity():
    import torch
    from distrain_b200 import cli
    built = []

    class FakeNode:
        def __init__(self, batch, node_id):
            self.batch, self.node_id = batch, node_id or "assigned-id"
            built.append((batch, self.node_id))

        def run(self, steps):
            if self.batch > 5:
                raise torch.cuda.OutOfMemoryError("fake")
            return [{"step": 1}]
    node, log = cli.run_with_oom_halving(FakeNode, 32, 10)
    assert [b for b, _ in built] == [32, 16, 8, 4] and node.batch == 4 and log == [{"step": 1}]
    assert {i for _, i in built} == {"assigned-id"}
    built.clear()

    class AlwaysOom(FakeNode):
        def run(self, steps):
            raise torch.cuda.OutOfMemoryError("fake")
    with pytest.raises(torch.cuda.OutOfMemoryError):
        cli.run_with_oom_halving(AlwaysOom, 4, 10)
    assert [b for b, _ in built] == [4, 2, 1]


def test_host_memory_pressure_rule():
    from distrain_b200.utils.resources import host_memory_fraction, memory_pressure
    assert 0.0 <= host_memory_fraction() <= 1.0
    assert memory_pressure(0.80, used_fraction=0.91) and not memory_pressure(0.80, used_fraction=0.89)
    assert not memory_pressure(0.95, used_fraction=0.999)  # threshold capped at 100 %


def test_calibration_probe_timeout_counts_as_not_fitting(monkeypatch):
    import subprocess as sp
    from distrain_b200 import cli

    def fake_run(cmd, **kw):
        assert kw["timeout"] == 300.0
        b = int(cmd[cmd.index("--batch-size") + 1])
        if b > 10:
            raise sp.TimeoutExpired(cmd, kw["timeout"])
        return sp.CompletedProcess(cmd, 0)
    monkeypatch.setattr(cli.subprocess, "run", fake_run)
    assert cli.calibrate_batch_size("ck", 128) == 10


def test_generate_with_byte_tokenizer(tmp_path):
    """generate --tokenizer bytes: the prompt's UTF-8 bytes (ids 3 + byte) and the decoded text."""
    from distrain_b200.config import ModelConfig
    from distrain_b200.models.params import ParamLayout, init_flat
    from distrain_b200.utils.checkpoint import save_safetensors
    cfg = ModelConfig(hidden_dim=32, num_layers=1, num_heads=4, num_kv_heads=2, ffn_hidden_dim=64, vocab_size=260,
                      max_seq_len=64)
    L = ParamLayout(cfg)
    ck = str(tmp_path / "m.safetensors")
    save_safetensors(L.to_state_dict(init_flat(L, seed=1)), ck)
    p = run(["generate", ck, "--prompt", "hi", "--tokenizer", "bytes", "--max-tokens", "3"])
    assert p.returncode == 0, p.stderr
    r = json.loads(p.stdout.strip().splitlines()[-1])
    assert r["ids"][:2] == [3 + ord("h"), 3 + ord("i")] and len(r["ids"]) == 5
    assert isinstance(r["text"], str) and r["text"].startswith("hi")

