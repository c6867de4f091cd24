"""Multi-node without a cluster: coordinator HTTP service + two CPU nodes (fp32 oracle model),
synthetic tokens, top-k 10% + INT8 deltas through the object store, pushes every few steps."""
import threading

import pytest
import torch

from distrain_b200.config import ModelConfig, CoordinatorConfig, CompressionConfig, OptimConfig
from distrain_b200.coordinator.service import CoordinatorService, bootstrap
from distrain_b200.parallel.http_node import HttpNode, adaptive_top_k
from distrain_b200.utils.storage import FsStore


def test_adaptive_top_k_reference_table():
    assert adaptive_top_k(25.0, None, 0) == 0.5 and adaptive_top_k(6.0, None, 0) == 0.75
    assert adaptive_top_k(4.0, None, 0) == 0.8
    assert abs(adaptive_top_k(4.0, 10, 1000) - 0.02) < 1e-9 and adaptive_top_k(4.0, 1, 10 ** 9) == 0.01


@pytest.mark.timeout(600)
def test_two_cpu_nodes_and_coordinator(tmp_path):
    cfg = ModelConfig(hidden_dim=64, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=128, vocab_size=512,
                      max_seq_len=128, rope_theta=10000.0)
    store = FsStore(str(tmp_path))
    bootstrap(store, cfg, seed=0)
    svc = CoordinatorService(CoordinatorConfig(min_contributions=0), store, flush_interval=3600)
    port = svc.start(host="127.0.0.1", port=0, threads=4)
    url = f"http://127.0.0.1:{port}"
    # a fixed small token pool makes the loss drop visibly within a few dozen steps
    pool = torch.randint(0, cfg.vocab_size, (8, 33), generator=torch.Generator().manual_seed(3), dtype=torch.int32)
    nodes = []
    for i in range(2):
        g = torch.Generator().manual_seed(10 + i)
        data = (lambda g=g: pool[torch.randint(0, 8, (4,), generator=g)])
        n = HttpNode(url, store, cfg, batch=4, seq_len=33, h_mini=5, optim=OptimConfig(lr=3e-3),
                     compression=CompressionConfig(top_k_fraction=0.1, quantize_int8=True), device="cpu",
                     node_id=f"cpu-node-{i}", data=data, poll_secs=0.2)
        n.register()
        nodes.append(n)
    th = [threading.Thread(target=n.run, args=(40,)) for n in nodes]
    for t in th:
        t.start()
    for t in th:
        t.join()
    svc.stop()
    assert not svc.last_error, svc.last_error
    assert all(not n.errors for n in nodes), [n.errors for n in nodes]
    assert svc.acc.state.checkpoint_version >= 2
    for n in nodes:
        assert any(p["accepted"] for p in n.pushes)
        first = sum(x["loss"] for x in n.log[:5]) / 5
        last = sum(x["loss"] for x in n.log[-5:]) / 5
        assert last < first, (first, last)
        assert n.version >= 1


def test_adaptive_push_mode():
    from distrain_b200.config import CompressionConfig
    from distrain_b200.parallel.compression import adaptive_push_mode
    cfg = CompressionConfig(top_k_fraction=0.1, quantize_int8=True, int8_block=256)
    assert adaptive_push_mode(False, 1e12, 400, 3.0, cfg) == ("topk", 0.1, 256)
    assert adaptive_push_mode(True, 0.0, 400, 6.0, cfg) == ("topk", 0.75, 256)   # no bandwidth yet: loss-based
    assert adaptive_push_mode(True, 100.0, 400, 3.0, cfg) == ("raw", 1.0, 0)     # 400 B within 10 s at 100 B/s
    kind, k, qb = adaptive_push_mode(True, 10.0, 4000, 3.0, cfg)                  # budget 100 B of 4000 raw
    assert kind == "topk" and qb == 0 and abs(k - 100 / 2000) < 1e-9


def test_loss_based_inner_lr_and_watchdog(tmp_path):
    """One CPU node with LR_MODE=loss_based: after the first-round warm-up every step's lr is
    lr_max * clamp(loss_ema / ln(vocab), 0.1, 1) of the losses before it; the watchdog stays quiet."""
    import math
    cfg = ModelConfig(hidden_dim=32, num_layers=1, num_heads=2, num_kv_heads=1, ffn_hidden_dim=64, vocab_size=256,
                      max_seq_len=64, rope_theta=10000.0)
    store = FsStore(str(tmp_path))
    bootstrap(store, cfg, seed=0)
    svc = CoordinatorService(CoordinatorConfig(min_contributions=0), store, flush_interval=3600)
    port = svc.start(host="127.0.0.1", port=0, threads=2)
    g = torch.Generator().manual_seed(5)
    n = HttpNode(f"http://127.0.0.1:{port}", store, cfg, batch=2, seq_len=17, h_mini=10, optim=OptimConfig(lr=1e-3),
                 compression=CompressionConfig(top_k_fraction=0.1), device="cpu", node_id="lr-node",
                 data=lambda: torch.randint(0, 256, (2, 17), generator=g, dtype=torch.int32), poll_secs=0.2,
                 loss_based_lr=True, expected_step_secs=1.0)
    n.register()
    n.run(25)
    svc.stop()
    assert not n.errors, n.errors
    warm = max(int(10 * 0.2), 2)
    ema = 0.0
    for i, row in enumerate(n.log):
        if i >= warm and ema > 0:
            want = 1e-3 * min(max(ema / math.log(256), 0.1), 1.0)
            assert abs(row["lr"] - want) < 1e-12, (i, row["lr"], want)
        ema = row["loss"] if i == 0 else ema * 0.9 + row["loss"] * 0.1
