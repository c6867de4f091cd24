"""train-box end to end on one GPU: the micro-test preset over local token shards, pushes every 10 steps
(one node merging its own deltas), JSONL log; the run must finish, merge, and report finite losses."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_train_box_micro_one_gpu(tmp_path):
    from distrain_b200.utils.data import prepare_random_shards
    data = tmp_path / "data"
    prepare_random_shards(str(data), num_shards=4, tokens_per_shard=200_000, vocab_size=32768)
    log = tmp_path / "log.jsonl"
    env = dict(os.environ, PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-m", "distrain_b200", "train-box", "--preset", "micro-test", "--steps", "40",
                        "--log-every", "20", "--push-every", "10", "--data-dir", str(data), "--output", str(log)],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    recs = [json.loads(line) for line in open(log)]
    assert [x["event"] for x in recs] == ["train_box_start", "train", "train", "train_box_done"]
    assert recs[0]["nodes"] == 1 and "4 of 4 shards" in recs[0]["data"]
    assert all(x["loss"] == x["loss"] and x["loss"] < 20 for x in recs[1:3])  # finite
    assert recs[-1]["steps"] == 40 and recs[-1]["version"] >= 1
