"""SM partition (green context) for the coordinator's merge: kernels on its stream stay on its SMs, write
the library's error word the host reads, and the merge run in it matches the merge on a normal stream."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _smids(stream, nblocks=2 * 148, spin_ns=200_000):
    from distrain_b200.ops import _lib
    L = _lib.lib()
    _lib.register("dt_smid_probe", [ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_void_p])
    out = torch.full((nblocks,), -1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    _lib.check(L.dt_smid_probe(out.data_ptr(), nblocks, spin_ns, stream.cuda_stream), "dt_smid_probe")
    stream.synchronize()
    ids = out.cpu()
    assert int(ids.min()) >= 0
    return set(ids.tolist())


def test_partition_confines_kernels_to_its_sms():
    from distrain_b200.parallel.partition import partition
    part = partition("cuda:0", 16)
    try:
        assert 16 <= part.sms < part.total_sms
        inside = _smids(part.stream)
        outside = _smids(torch.cuda.Stream())
        assert len(inside) <= part.sms, (len(inside), part.sms)
        assert len(outside) > part.sms
    finally:
        part.close()


def test_partition_kernels_write_the_error_word_the_host_reads():
    from distrain_b200 import ops
    from distrain_b200.ops import _lib
    from distrain_b200.parallel.partition import partition
    L = _lib.lib()
    _lib.register("dt_raise_error", [ctypes.c_int, ctypes.c_void_p])
    part = partition("cuda:0", 8)
    try:
        ops.clear_device_error()
        _lib.check(L.dt_raise_error(777, part.stream.cuda_stream), "dt_raise_error")
        part.stream.synchronize()
        code, site = ops.device_error()
        assert (code, site) == (6, 777)
    finally:
        ops.clear_device_error()
        part.close()


def test_distributed_merge_in_partition_matches_whole_gpu():
    """The one-node distributed merge (range, apply, broadcast, completion wait) run on a 16-SM partition
    gives the weights of the same merge on an ordinary stream."""
    from distrain_b200.config import CompressionConfig
    from distrain_b200.parallel.compression import DeviceCompressor
    from distrain_b200.parallel.merge import DistributedMerger, Contribution
    from distrain_b200.config import ModelConfig
    from distrain_b200.models.params import ParamLayout
    from distrain_b200.parallel.partition import partition
    L = ParamLayout(ModelConfig(hidden_dim=64, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=128,
                                vocab_size=512))
    dev = torch.device("cuda")
    torch.manual_seed(5)
    theta0 = torch.randn(L.total, device=dev) * 0.02
    cfg = CompressionConfig(top_k_fraction=0.2, quantize_int8=True, int8_block=256)
    contribs, stats, keep = [], [], []
    for i, sc in enumerate([1.0, 3.0]):
        comp = DeviceCompressor(L, dev, cfg)
        comp.snap.copy_(theta0)
        comp.begin(theta0 - torch.randn(L.total, device=dev) * 1e-3 * sc)
        comp.finish()
        torch.cuda.synchronize()
        st = comp.read_stats()
        K = st["num_params_kept"]
        stats.append(st["wire"])
        p = comp.payload
        keep.append(comp)
        contribs.append(Contribution(idx_ptr=p.idx.data_ptr(), q_ptr=p.q.data_ptr(), val_ptr=p.val.data_ptr(),
                                     scales_ptr=p.scales.data_ptr(), win_ptr=p.win.data_ptr(), count=K, block=256,
                                     dense=False, weight=1000.0 / (i + 1)))
    results = []
    part = partition(dev, 16)
    try:
        for stream in (torch.cuda.Stream(priority=-100), part.stream):
            theta = theta0.clone()
            ctl = torch.zeros(DistributedMerger.CTL_BYTES, dtype=torch.uint8, device=dev)
            dm = DistributedMerger(0, 1, L.total, dev, theta, [theta.data_ptr()], 0, ctl, [ctl.data_ptr()],
                                   stream=stream)
            torch.cuda.synchronize()
            info = dm.run_local(contribs, stats, 1.0, 1)
            assert info["accepted"] == 2
            torch.cuda.synchronize()
            results.append(theta.clone())
    finally:
        part.close()
    # the scatter-add order of overlapping entries depends on the grid, so the two agree to rounding
    assert not torch.equal(results[0], theta0)
    assert torch.allclose(results[0], results[1], atol=1e-7, rtol=1e-6)
