"""Every cross-GPU wait in the kernel library is bounded: a wait on a flag that nothing sets gives up after
its limit, records an error code and site in the library's error word, skips its work and returns, and
the CUDA context stays usable (no trap, no fault, no hang). Both tests make a wait run out on purpose,
on a single GPU, with counters that stay zero."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from distrain_b200 import ops
    return ops


def test_cross_node_wait_times_out_and_reports():
    import ctypes
    from distrain_b200.ops._lib import lib, register, check, c_void, c_int
    ops = _ops()
    register("dt_dm_wait", [c_void, ctypes.c_ulonglong, c_int, ctypes.c_ulonglong, c_void])
    ops.clear_device_error()
    counter = torch.zeros(8, dtype=torch.int64, device="cuda")  # never incremented
    s = torch.cuda.Stream()
    check(lib().dt_dm_wait(counter.data_ptr(), 1, 977, 200_000_000, s.cuda_stream), "dt_dm_wait")  # 0.2 s
    s.synchronize()
    code, site = ops.device_error(s)
    assert (code, site) == (4, 977)  # DT_ERR_TIMEOUT_PEER at the caller's site
    ops.clear_device_error(s)
    # the context is fine: a satisfied wait returns at once and ordinary work runs
    check(lib().dt_dm_wait(counter.data_ptr(), 0, 978, 200_000_000, s.cuda_stream), "dt_dm_wait")
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float((x * 2).sum()) == 2 * 1023 * 1024 / 2
    s.synchronize()
    assert ops.device_error(s)[0] == 0


def test_tensor_parallel_norm_skips_work_when_the_peer_partial_never_arrives():
    ops = _ops()
    ops.clear_device_error()
    M, H = 64, 256
    x = torch.randn(M, H, device="cuda")
    br = torch.randn(M, H, device="cuda").bfloat16()
    br2 = torch.zeros(M, H, device="cuda", dtype=torch.bfloat16)  # the "peer" buffer nobody fills
    w = torch.ones(H, device="cuda")
    y = torch.full((M, H), float("nan"), device="cuda", dtype=torch.bfloat16)
    rstd = torch.full((M,), -1.0, device="cuda")
    out = torch.full((M, H), -7.0, device="cuda")
    counters = torch.zeros(1024, dtype=torch.int32, device="cuda")  # arrivals @0, consumed @128 B, done @256 B
    base = counters.data_ptr()
    ops.add_rmsnorm_fwd_tp(x=x, br=br, br2=br2, w=w, y=y, rstd=rstd, eps=1e-5, M=M, H=H, arrivals=base,
                           consumed=base + 128, done_blocks=base + 256, out_resid=out)
    torch.cuda.synchronize()
    code, site = ops.device_error()
    assert (code, site) == (4, 900)
    # the blocks gave up instead of reading a partial that never came
    assert bool(torch.isnan(y.float()).all()) and bool((rstd == -1.0).all()) and bool((out == -7.0).all())
    ops.clear_device_error()
    # and the same kernel without a peer partial runs normally afterwards
    ops.add_rmsnorm_fwd(x=x, br=br, w=w, out_resid=out, y=y, rstd=rstd, eps=1e-5, M=M, H=H)
    torch.cuda.synchronize()
    r = x + br.float()
    want = r * torch.rsqrt((r * r).mean(-1, keepdim=True) + 1e-5)
    assert torch.allclose(y.float(), want, atol=3e-2, rtol=2e-2)
    assert ops.device_error()[0] == 0
