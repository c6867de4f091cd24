"""Roofline arithmetic used in the benchmark JSON lines."""
from distrain_b200.config import preset
from distrain_b200.roofline import distributed_merge_roofline, peaks, step_roofline, train_flops_per_token


def test_flops_per_token_and_fraction():
    cfg = preset("tiny")
    n = cfg.param_count()
    f = train_flops_per_token(cfg, 1024)
    assert f == 6 * n + 6 * cfg.num_layers * 1024 * cfg.hidden_dim
    assert train_flops_per_token(cfg, 1024, act_ckpt=True) == f + 2 * (n - cfg.vocab_size * cfg.hidden_dim)
    pk = {"hbm_gbs": 6000.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0, "src": "test"}
    r = step_roofline(cfg, 1024, 1e6, 2, pk=pk)
    assert abs(r["model_tflops_per_gpu"] - f * 1e6 / 2 / 1e12) < 0.1
    assert abs(r["frac_of_test_sustained_bf16"] - r["model_tflops_per_gpu"] / 1400.0) < 1e-3
    assert set(peaks()) >= {"hbm_gbs", "bf16_tflops", "bf16_tflops_sustained", "src"}


def test_distributed_merge_bytes():
    pk = {"hbm_gbs": 1000.0, "bf16_tflops": 1.0, "bf16_tflops_sustained": 1.0, "src": "t"}
    n, P, W = 1_000_000, 4_000_000.0, 4
    r = distributed_merge_roofline(n, P, W, merge_ms=10.0, pk=pk)
    s = n * 4 / W
    assert r["nvlink_bytes_per_gpu"] == int((W - 1) * (P / W + s))
    assert r["hbm_bytes_per_gpu"] == int(2 * s + P + (W - 1) * s)
    one = distributed_merge_roofline(n, P, 1, merge_ms=1.0, pk=pk)
    assert one["nvlink_bytes_per_gpu"] == 0 and one["bound"] == "hbm"
