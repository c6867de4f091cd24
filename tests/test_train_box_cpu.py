"""train-box command pieces that need no GPU: run-config overrides, per-node batch sources (the
reference's deterministic shard assignment over local shards, or seeded synthetic tokens), the pinned
batch feed of the end-to-end loop, and the command's argument parser."""
import argparse
import os

import numpy as np
import pytest
import torch

from distrain_b200 import cli
from distrain_b200.config import bench_config
from distrain_b200.parallel.launch import node_batches, node_layout
from distrain_b200.parallel.node import BatchFeed
from distrain_b200.utils.data import prepare_random_shards
from distrain_b200.utils.native import shard_assignment


def _args(**kw):
    base = dict(push_every=None, tp=None, checkpoint_store=None, checkpoint_every=None, keep_versions=None,
                metrics_port=None, watchdog_secs=None, swap_mode=None, ef_on_swap=None, seed=None, payload_slots=None,
                resume=False, loss_based_lr=False, bandwidth_adaptive=False, reset_optimizer=False,
                activation_checkpointing=False, top_k=None, no_int8=False, lr=None, batch_size=None, seq_len=None,
                grad_accum=None)
    base.update(kw)
    return argparse.Namespace(**base)


def test_overrides_touch_only_the_given_fields():
    ref = bench_config("tiny")
    run = cli.apply_run_overrides(bench_config("tiny"), _args())
    assert run.to_dict() == ref.to_dict()
    run = cli.apply_run_overrides(bench_config("tiny"), _args(push_every=7, top_k=0.25, no_int8=True, lr=1e-3,
                                                              checkpoint_store="/tmp/x", checkpoint_every=3,
                                                              resume=True, swap_mode="push_partial",
                                                              reset_optimizer=True, seq_len=2048, batch_size=3))
    assert (run.push_every, run.compression.top_k_fraction, run.compression.quantize_int8) == (7, 0.25, False)
    assert (run.optim.lr, run.checkpoint_store, run.checkpoint_every, run.resume) == (1e-3, "/tmp/x", 3, True)
    assert (run.swap_mode, run.reset_optimizer_on_swap, run.micro_batch, run.seq_len) == ("push_partial", True, 3, 2048)
    assert run.model.max_seq_len >= 2048


def test_node_layout():
    assert node_layout(8, 1) == (1, 8)
    assert node_layout(8, 2) == (2, 4)
    assert node_layout(1, 2) == (1, 1)  # tensor parallelism needs at least T ranks
    assert node_layout(6, 4) == (1, 6)


def test_synthetic_source_is_seeded_per_node():
    run = bench_config("micro-test")
    a0, _ = node_batches(run, 0, 4)
    a0b, _ = node_batches(run, 0, 4)
    a1, _ = node_batches(run, 1, 4)
    x, y, z = a0(), a0b(), a1()
    assert x.shape == (run.micro_batch, run.seq_len) and x.dtype == torch.int32
    assert torch.equal(x, y) and not torch.equal(x, z)
    assert int(x.max()) < run.model.vocab_size and int(x.min()) >= 0


def test_shard_source_reads_the_nodes_assigned_shards(tmp_path):
    run = bench_config("micro-test")
    run.micro_batch, run.seq_len = 2, 16
    prepare_random_shards(str(tmp_path), num_shards=10, tokens_per_shard=4096, vocab_size=run.model.vocab_size)
    shards = [np.fromfile(os.path.join(tmp_path, f"shard_{i:04d}.bin"), dtype="<u2") for i in range(10)]
    for node in range(4):
        src, desc = node_batches(run, node, 4, str(tmp_path), shards_fraction=0.2)
        want = shard_assignment(f"box-node-{node}", 0, 10, 2)
        assert len(want) == 2 and f"2 of 10 shards" in desc
        b = src()
        assert b.shape == (2, 16) and b.dtype == torch.int32
        first = shards[want[0]]
        assert torch.equal(b.flatten().long(), torch.from_numpy(first[:32].astype(np.int64)))
    # one node reads every shard
    src, desc = node_batches(run, 0, 1, str(tmp_path))
    assert "10 of 10" in desc
    with pytest.raises(FileNotFoundError):
        node_batches(run, 0, 1, _empty(tmp_path))


def _empty(tmp_path):
    d = tmp_path / "empty"
    d.mkdir()
    return str(d)


def test_batch_feed_round_robin_and_shape_check():
    n = [0]

    def src():
        n[0] += 1
        return torch.full((2, 3), n[0], dtype=torch.int32)
    feed = BatchFeed(src, 2, 3, depth=3)
    assert len(feed) == 3
    got = [feed[i % len(feed)] for i in range(5)]
    # elements are the buffers themselves: buffers 0 and 1 were refilled by the reads of steps 3 and 4
    assert [int(g[0, 0]) for g in got] == [4, 5, 3, 4, 5]
    assert got[0] is feed.bufs[0] and feed.fetched == 5
    bad = BatchFeed(lambda: torch.zeros(1, 3, dtype=torch.int32), 2, 3)
    with pytest.raises(ValueError):
        bad[0]


def test_batch_feed_gathers_the_micro_batches_of_a_step():
    """With gradient accumulation a step's buffer holds `accum` consecutive source batches."""
    n = [0]

    def src():
        n[0] += 1
        return torch.full((2, 3), n[0], dtype=torch.int32)
    feed = BatchFeed(src, 2, 3, depth=2, accum=3)
    b = feed[0]
    assert b.shape == (6, 3) and feed.fetched == 3
    assert [int(b[r, 0]) for r in range(6)] == [1, 1, 2, 2, 3, 3]
    run = cli.apply_run_overrides(bench_config("tiny"), _args(grad_accum=4))
    assert run.grad_accum_steps == 4 and run.micro_batch == 32


def test_train_box_parser():
    with pytest.raises(SystemExit) as e:
        cli.main(["train-box", "--help"])
    assert e.value.code == 0


def test_node_data_position_survives_a_restart(tmp_path):
    """train-box keeps each node's data position in the checkpoint store; a resumed node continues."""
    from distrain_b200.parallel.launch import restore_data_state, save_data_state
    from distrain_b200.utils.storage import FsStore
    store = FsStore(str(tmp_path / "ck"))
    run = bench_config("micro-test")
    run.micro_batch, run.seq_len = 2, 16
    prepare_random_shards(str(tmp_path / "d"), num_shards=3, tokens_per_shard=2048, vocab_size=run.model.vocab_size)
    for data_dir in (str(tmp_path / "d"), None):
        a, _ = node_batches(run, 1, 2, data_dir, shards_fraction=0.5)
        for _ in range(40):
            a()
        assert save_data_state(store, 1, a)
        want = a()
        b, _ = node_batches(run, 1, 2, data_dir, shards_fraction=0.5)
        assert restore_data_state(store, 1, b)
        assert torch.equal(b(), want)
    c, _ = node_batches(run, 0, 2, None)
    assert not restore_data_state(store, 0, c)  # nothing stored for node 0
