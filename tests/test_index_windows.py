"""Compressed payloads over flat buffers larger than 2^31 elements: kept indices are stored relative to
2^31-element windows and the payload records where each window starts.

CPU: chunk tables never straddle a window boundary. GPU: a ~2.2 G-parameter layout with values planted
on both sides of the 2^31 boundary compresses to the right flat indices and merges into the right
checkpoint entries."""

import pytest
import torch


class _Entry:
    def __init__(self, name, offset, numel):
        self.name, self.offset, self.numel, self.shape = name, offset, numel, (numel,)


class _Layout:
    """Minimal ParamLayout stand-in: two tensors whose second one starts just below 2^31."""
    from distrain_b200.models.params import ParamLayout as _PL
    WINDOW = _PL.WINDOW
    chunk_tables = _PL.chunk_tables

    def __init__(self, n0, n1):
        self.entries = [_Entry("a", 0, n0), _Entry("b", (n0 + 3) // 4 * 4, n1)]
        self.total = (self.entries[1].offset + n1 + 3) // 4 * 4

    def num_params(self):
        return sum(e.numel for e in self.entries)


def test_chunks_split_at_windows():
    W = 1 << 31
    L = _Layout(W - 1000, 1 << 20)
    cseg, cs, ce, nseg = L.chunk_tables("cpu")
    assert nseg == 2
    for s, e in zip(cs.tolist(), ce.tolist()):
        assert s // W == (e - 1) // W, (s, e)
    assert ce[-1] == L.entries[1].offset + L.entries[1].numel
    # chunks tile every tensor
    assert int((ce - cs).sum()) == L.num_params()


@pytest.mark.gpu
def test_windowed_payload_and_merge():
    from distrain_b200.config import CompressionConfig
    from distrain_b200.parallel.compression import DeviceCompressor
    from distrain_b200.parallel.merge import DeviceMerger, Contribution
    W = 1 << 31
    dev = torch.device("cuda")
    L = _Layout(W - 4096, 300_000)
    n = L.total
    comp = DeviceCompressor(L, dev, CompressionConfig(top_k_fraction=1e-4, quantize_int8=False,
                                                      per_tensor_adaptive=False))
    assert comp.nwin == 2
    g = torch.Generator(device="cuda").manual_seed(3)
    # small noise everywhere, large planted values around the boundary and at the far ends
    comp.snap.normal_(0.0, 1e-6, generator=g)
    planted = torch.tensor([5, 1234567, W - 4100, W - 1, W, W + 7, n - 5], device=dev, dtype=torch.int64)
    comp.snap[planted] = torch.linspace(1.0, 2.0, planted.numel(), device=dev)
    comp.ef.zero_()
    master = torch.zeros(n, device=dev)
    delta = comp.snap.clone()
    comp.begin(master)
    comp.finish()
    torch.cuda.synchronize()
    st = comp.read_stats()
    K = st["num_params_kept"]
    p = comp.payload
    gi = p.global_indices(K)
    assert int(p.win[1]) > 0 and int(p.win[2]) == 2 ** 63 - 1
    assert bool((gi[1:] > gi[:-1]).all()), "flat indices ascending"
    assert bool((gi < n).all())
    torch.testing.assert_close(p.val[:K], delta[gi], rtol=0, atol=0)
    kept = set(gi.tolist())
    assert all(int(i) in kept for i in planted.tolist())
    del delta
    # merge the payload in place into a zero checkpoint: theta[gi] = -coef * val
    theta = torch.zeros(n, device=dev)
    m = DeviceMerger(n, dev, theta_buffer=theta)
    c = Contribution(idx_ptr=p.idx.data_ptr(), q_ptr=0, val_ptr=p.val.data_ptr(), scales_ptr=0, count=K, block=0,
                     dense=False, weight=1.0, win_ptr=p.win.data_ptr())
    dst = torch.zeros(n, device=dev)
    torch.cuda.synchronize()  # the merger's stream does not wait for the default stream's fills
    m.accumulate_apply([c], [1.0], 1.0, stage32=[dst.data_ptr()])
    m.stream.synchronize()
    torch.testing.assert_close(theta[gi], -p.val[:K], rtol=0, atol=0)
    assert float(theta.abs().sum()) == pytest.approx(float(p.val[:K].abs().double().sum()), rel=1e-5)
    diff = (dst != theta).nonzero().flatten()
    assert diff.numel() == 0, (f"{diff.numel()} broadcast mismatches, first {diff[:4].tolist()} last "
                               f"{diff[-4:].tolist()}; dst {dst[diff[:4]].tolist()} theta {theta[diff[:4]].tolist()}")
