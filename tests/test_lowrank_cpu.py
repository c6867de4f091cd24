"""Low-rank delta compression (the reference's rank-r option, kept as its negative result): exact recovery
of a rank-r delta, orthonormal range basis, 1-D passthrough, and error feedback carrying the residual."""
import torch

from distrain_b200.parallel.lowrank import compress_lowrank, decompress_lowrank, truncated_svd


def test_rank_r_delta_is_recovered_and_basis_is_orthonormal():
    g = torch.Generator().manual_seed(0)
    m, n, r = 64, 48, 4
    d = (torch.randn(m, r, generator=g) @ torch.randn(r, n, generator=g)).reshape(-1)
    u, v = truncated_svd(d, m, n, r)
    q = u.double()
    torch.testing.assert_close(q.t() @ q, torch.eye(r, dtype=torch.float64), atol=1e-5, rtol=0)
    rec = (u.double() @ v.double().t()).reshape(-1).float()
    assert float((rec - d).norm() / d.norm()) < 1e-4


def test_roundtrip_passthrough_and_error_feedback():
    g = torch.Generator().manual_seed(1)
    delta = {"w": torch.randn(32 * 40, generator=g), "b": torch.randn(40, generator=g)}
    shapes = {"w": [32, 40], "b": [40]}
    ef = {}
    lr, stats = compress_lowrank(delta, shapes, 8, ef)
    out = decompress_lowrank(lr)
    assert torch.equal(out["b"], delta["b"]) and "b" not in ef          # 1-D tensors pass through exactly
    torch.testing.assert_close(out["w"] + ef["w"], delta["w"], atol=1e-5, rtol=0)  # sent + residual = delta
    assert 0.0 < stats["reconstruction_error"] < 1.0 and stats["compression_ratio"] > 1.0
    # the next round adds the residual back before compressing
    lr2, _ = compress_lowrank({"w": torch.zeros(32 * 40), "b": torch.zeros(40)}, shapes, 8, ef)
    out2 = decompress_lowrank(lr2)
    assert float(out2["w"].norm()) > 0.0


def test_native_test_matrix_equals_the_draw_by_draw_loop():
    from distrain_b200.parallel.lowrank import _omega, _omega_loop
    for m, n, r in [(64, 48, 4), (768, 256, 8), (3, 5, 2)]:
        a, b = _omega(m, n, r), _omega_loop(m, n, r)
        assert a.shape == b.shape == (n, r)
        assert torch.equal(a, b)  # the same libm on both sides
