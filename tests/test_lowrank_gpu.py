"""Low-rank compression of CUDA deltas runs on the GPU and gives the CPU result (same test matrix, float64
range finder), with the residual kept in a device error buffer."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_lowrank_on_device_matches_host():
    from distrain_b200.parallel.lowrank import compress_lowrank, decompress_lowrank
    g = torch.Generator().manual_seed(3)
    delta = {"w": torch.randn(96 * 64, generator=g), "b": torch.randn(64, generator=g)}
    shapes = {"w": [96, 64], "b": [64]}
    ef_h, ef_d = {}, {}
    lr_h, st_h = compress_lowrank(delta, shapes, 8, ef_h)
    lr_d, st_d = compress_lowrank({k: v.cuda() for k, v in delta.items()}, shapes, 8, ef_d)
    assert ef_d["w"].is_cuda
    out_h, out_d = decompress_lowrank(lr_h), decompress_lowrank(lr_d)
    torch.testing.assert_close(out_d["w"], out_h["w"], atol=1e-5, rtol=1e-5)
    assert torch.equal(out_d["b"], out_h["b"])
    torch.testing.assert_close(ef_d["w"].cpu(), ef_h["w"], atol=1e-5, rtol=1e-5)
    assert st_d["reconstruction_error"] == pytest.approx(st_h["reconstruction_error"], rel=1e-6)
