"""The per-rank device-memory estimate against what the B200 runs measured (bench.py
device_memory_used_gb_max): tiny 17.6 GB, small 85.2 GB (bandwidth-adaptive), large TP=2 188.3 GB."""
from distrain_b200.config import bench_config
from distrain_b200.memory import check_fits, estimate_rank_bytes


def test_estimates_track_measurements():
    for name, n_nodes, measured, tol in (("tiny", 1, 17.6e9, 0.15), ("small", 2, 85.2e9, 0.10),
                                         ("large", 4, 188.3e9, 0.05)):
        est = estimate_rank_bytes(bench_config(name), n_nodes)["total"]
        assert abs(est - measured) <= tol * measured and est <= measured, (name, est / 1e9)


def test_every_preset_fits_a_b200_as_configured():
    b200 = 183359 * 2 ** 20  # nvidia-smi total
    for name in ("micro", "tiny", "small", "medium", "large"):
        fits, est = check_fits(bench_config(name), b200, n_nodes=4)
        assert fits, (name, est["total"] / 1e9)
