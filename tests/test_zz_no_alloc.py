"""The allocation-free compression entry point (``dt_compress_noalloc``), called through its exported C
symbol, against the regular entry points (caller-allocated workspace) on two consecutive pushes.

It serves callers that cannot allocate device memory (their device memory belongs to their own
allocator, or they must not allocate once running): they pass inputs and outputs only and the
pipeline's scratch lives in a fixed array inside the library. Collected last on purpose."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _sym():
    from distrain_b200.ops import _lib
    L = _lib.lib()
    f = L.dt_compress_noalloc
    v, i, ll, fl = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float
    f.argtypes = [v, v, v, v, v, v, i, i, v, ll, fl, i, v, v, v, v, i, ll, v, v]
    f.restype = ctypes.c_int
    L.dt_compress_noalloc_scratch_bytes.restype = ll
    L.dt_compress_noalloc_min_capacity.argtypes = [ll, i, fl]
    L.dt_compress_noalloc_min_capacity.restype = ll
    return f, L


def test_noalloc_matches_allocating_entry_point_twice():
    from distrain_b200.config import ModelConfig, CompressionConfig
    from distrain_b200.models.params import ParamLayout
    from distrain_b200.parallel.compression import DeviceCompressor, DevicePayload
    f, L = _sym()
    assert L.dt_compress_noalloc_scratch_bytes() == 32 << 20
    dev = torch.device("cuda")
    cfg = ModelConfig(hidden_dim=128, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=256, vocab_size=1024)
    layout = ParamLayout(cfg)
    cc = CompressionConfig(top_k_fraction=0.1, quantize_int8=True, per_tensor_adaptive=True, int8_block=256)
    torch.manual_seed(0)
    mask = torch.zeros(layout.total, dtype=torch.bool, device=dev)
    for e in layout.entries:
        mask[e.offset:e.offset + e.numel] = True

    ref = DeviceCompressor(layout, dev, cc)          # regular path: workspace allocated by the caller
    snap0 = torch.randn(layout.total, device=dev) * mask
    ref.snap.copy_(snap0)
    snap = snap0.clone()
    ef = torch.zeros(layout.total, device=dev)
    cap = ref.capacity
    out = DevicePayload.allocate(cap, 256, dev)
    stats = torch.zeros(ref.stats_dev.numel(), dtype=torch.float64, device=dev)
    stream = torch.cuda.current_stream().cuda_stream

    for call in range(2):
        master = snap0 - torch.randn(layout.total, device=dev) * 1e-3 * (call + 1) * mask
        ref.begin(master)
        ref.finish()
        rc = f(master.data_ptr(), snap.data_ptr(), ef.data_ptr(), ref.cseg.data_ptr(), ref.cstart.data_ptr(),
               ref.cend.data_ptr(), ref.nchunks, ref.nseg, ref.seg_len.data_ptr(), layout.total, 0.1, 1,
               out.idx.data_ptr(),
               out.val.data_ptr(), out.q.data_ptr(), out.scales.data_ptr(), 256, cap, stats.data_ptr(), stream)
        assert rc == 0
        torch.cuda.synchronize()
        k_ref = int(ref.stats_host[ref.nseg * 6].item())
        k = int(stats[ref.nseg * 6].item())
        assert k == k_ref and k > 0
        p = ref.payload
        assert torch.equal(out.idx[:k], p.idx[:k])
        assert torch.allclose(out.val[:k], p.val[:k], rtol=0, atol=0)
        assert torch.equal(out.q[:k], p.q[:k])
        nb = (k + 255) // 256
        assert torch.allclose(out.scales[:nb], p.scales[:nb], rtol=1e-6, atol=0)
        assert torch.equal(ef, ref.ef) and torch.equal(snap, ref.snap)
        assert torch.allclose(stats.cpu(), ref.stats_host, rtol=1e-9, atol=0)
        snap0 = master.clone()

    from distrain_b200 import ops
    assert ops.device_error()[0] == 0


def test_noalloc_rejects_oversized_problem():
    f, L = _sym()
    s = torch.cuda.current_stream().cuda_stream
    big_nseg = 1 << 16  # histograms alone would exceed the 32 MiB scratch
    n = 1 << 20
    rc = f(None, None, None, None, None, None, 1, big_nseg, None, n, 0.1, 1, None, None, None, None, 256, n, None, s)
    assert rc == -20
    # 2^31 elements or more: 32-bit flat indices cannot address them
    big = 1 << 31
    rc = f(None, None, None, None, None, None, 1, 4, None, big, 0.1, 1, None, None, None, None, 256, big, None, s)
    assert rc == -22
    # output arrays shorter than the largest possible selection
    need = L.dt_compress_noalloc_min_capacity(n, 4, 0.1)
    assert need == -(-n // 10) + 4
    rc = f(None, None, None, None, None, None, 1, 4, None, n, 0.1, 1, None, None, None, None, 256, need - 1, None, s)
    assert rc == -23
    # invalid arguments
    for nseg, nchunks, nel, k in ((0, 1, n, 0.1), (4, 0, n, 0.1), (4, 1, 0, 0.1), (4, 1, n, 0.0), (4, 1, n, 1.5)):
        rc = f(None, None, None, None, None, None, nchunks, nseg, None, nel, k, 1, None, None, None, None, 256, n,
               None, s)
        assert rc == -10
