"""Fused compression and peer-pull merge kernels vs the CPU restatement of the reference algorithms."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _layout():
    from distrain_b200.config import ModelConfig
    from distrain_b200.models.params import ParamLayout
    cfg = ModelConfig(hidden_dim=64, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=128, vocab_size=512)
    return ParamLayout(cfg)


@pytest.mark.parametrize("k_fraction,adaptive,flat", [(0.1, True, False), (0.01, True, False), (0.99, True, False),
                                                      (0.1, False, False), (0.1, True, True), (0.3, False, True)])
def test_device_compress_matches_reference(k_fraction, adaptive, flat):
    """flat: the largest tensor's deltas all have one magnitude, so a whole 32768-element chunk falls in the
    boundary bin - more than a chunk's candidate slot holds - and the selection takes the full-buffer
    passes; ties are broken by ascending index as in the reference."""
    from distrain_b200.config import CompressionConfig
    from distrain_b200.parallel.compression import DeviceCompressor, sparsify_topk, quantize_int8
    L = _layout()
    dev = torch.device("cuda")
    torch.manual_seed(0)
    cfg = CompressionConfig(top_k_fraction=k_fraction, quantize_int8=True, per_tensor_adaptive=adaptive, int8_block=256)
    comp = DeviceCompressor(L, dev, cfg)
    snap = torch.zeros(L.total, device=dev)
    mask = torch.zeros(L.total, dtype=torch.bool, device=dev)
    for e in L.entries:
        mask[e.offset:e.offset + e.numel] = True
    delta = torch.randn(L.total, device=dev) * 1e-3 * mask
    # per-tensor scale variety so the adaptive budget matters; a few exact ties
    for i, e in enumerate(L.entries):
        delta[e.offset:e.offset + e.numel] *= (1 + i % 5)
    delta[L.entries[3].offset:L.entries[3].offset + 8] = 0.5
    ef0 = torch.randn(L.total, device=dev) * 1e-4 * mask
    if flat:
        big = max(L.entries, key=lambda e: e.numel)
        sl = slice(big.offset, big.offset + big.numel)
        delta[sl] = torch.where(torch.rand(big.numel, device=dev) < 0.5, -2e-3, 2e-3)
        ef0[sl] = 0.0
    comp.snap.copy_(snap)
    comp.ef.copy_(ef0)
    master = snap - delta
    comp.begin(master)
    comp.finish()
    torch.cuda.synchronize()
    st = comp.read_stats()
    K = st["num_params_kept"]
    p = comp.payload
    idx = p.idx[:K].long().cpu()
    vals = p.val[:K].cpu()
    combined = (delta + ef0).cpu()
    # reference selection per tensor
    dd = {e.name: combined[e.offset:e.offset + e.numel] for e in L.entries}
    _, ridx, rvals = sparsify_topk(dd, k_fraction, adaptive)
    ref_idx = torch.cat([ridx[e.name] + e.offset for e in L.entries])
    ref_val = torch.cat([rvals[e.name] for e in L.entries])
    assert torch.equal(idx, ref_idx)
    assert torch.equal(vals, ref_val)
    assert torch.all(idx[1:] > idx[:-1])
    # error feedback residual: combined with kept entries zeroed
    ref_ef = combined.clone()
    ref_ef[ref_idx] = 0
    assert torch.equal(comp.ef.cpu(), ref_ef)
    # snapshot refreshed to master
    assert torch.equal(comp.snap, master)
    # int8 blocks of 256 over the kept stream
    q, sc = quantize_int8(ref_val, 256)
    assert torch.equal(p.q[:K].cpu(), q)
    assert torch.allclose(p.scales[:sc.numel()].cpu(), sc)
    assert abs(st["dense_norm"] - float(combined.double().norm())) < 1e-6 * max(1, st["dense_norm"])
    # statistics of the dequantised values as sent (what the coordinator validates and clips on)
    deq = q.float() * sc[torch.arange(K) // 256]
    ss, mx, nf = st["wire"]
    assert abs(ss - float((deq.double() ** 2).sum())) < 1e-5 * ss
    assert mx == pytest.approx(float(deq.abs().max()), rel=1e-6) and nf == 0


def test_compress_short_capacity_writes_nothing_past_it():
    """A capacity below the selection: entries beyond it are not written (sentinels past the capacity
    survive), they stay in error feedback, and the device error word reports an out-of-bounds condition."""
    from distrain_b200.config import CompressionConfig
    from distrain_b200.parallel.compression import DeviceCompressor, DevicePayload
    from distrain_b200 import ops
    from distrain_b200.ops._lib import check, stream_ptr
    L = _layout()
    dev = torch.device("cuda")
    torch.manual_seed(1)
    cfg = CompressionConfig(top_k_fraction=0.1, quantize_int8=True, per_tensor_adaptive=True, int8_block=256)
    comp = DeviceCompressor(L, dev, cfg)
    full = comp.capacity
    short = full // 2
    p = DevicePayload.allocate(full, 256, dev)
    p.idx.fill_(-7)
    p.val.fill_(123.0)
    p.q.fill_(77)
    mask = torch.zeros(L.total, dtype=torch.bool, device=dev)
    for e in L.entries:
        mask[e.offset:e.offset + e.numel] = True
    delta = torch.randn(L.total, device=dev) * 1e-3 * mask
    comp.snap.zero_()
    comp.ef.zero_()
    ops.clear_device_error()
    comp.begin(-delta)
    check(comp.L.dt_compress_finish(comp.ef.data_ptr(), comp.cseg.data_ptr(), comp.cstart.data_ptr(),
                                    comp.cend.data_ptr(), comp.nchunks, comp.nseg, comp.ws.data_ptr(), 0.1, 1,
                                    p.idx.data_ptr(), p.val.data_ptr(), p.q.data_ptr(), p.scales.data_ptr(), 256,
                                    short, comp.win_chunk.data_ptr(), comp.nwin, p.win.data_ptr(), stream_ptr()),
          "dt_compress_finish")
    torch.cuda.synchronize()
    code, site = ops.device_error()
    ops.clear_device_error()
    assert code == 5 and site == 710
    assert torch.all(p.idx[short:] == -7) and torch.all(p.val[short:] == 123.0) and torch.all(p.q[short:] == 77)
    kept = p.idx[:short].long()
    assert bool((kept >= 0).all()) and torch.all(kept[1:] > kept[:-1])
    # written entries left error feedback; the selected-but-unwritten ones (and the unselected) stay there
    written = torch.zeros(L.total, dtype=torch.bool, device=dev)
    written[kept] = True
    assert torch.all(comp.ef[written] == 0)
    assert torch.equal(comp.ef[~written], delta[~written])


@pytest.mark.parametrize("momentum,in_place", [(0.0, True), (0.0, False), (0.9, False)])
def test_device_merge_matches_reference(momentum, in_place):
    """Merge of three compressed payloads (one an outlier that gets clipped) against the fp32 reference
    merge: in place into a staging-style buffer, into a private copy, and with Nesterov momentum."""
    from distrain_b200.config import CompressionConfig
    from distrain_b200.parallel.compression import DeviceCompressor, dequantize_int8
    from distrain_b200.parallel.merge import DeviceMerger, Contribution, merge_reference
    L = _layout()
    dev = torch.device("cuda")
    torch.manual_seed(1)
    theta = torch.randn(L.total, device=dev) * 0.02
    cfg = CompressionConfig(top_k_fraction=0.2, quantize_int8=True, int8_block=256)
    contribs, dense_deltas, weights = [], [], []
    keep = []
    scales_norm = [1.0, 1.0, 10.0]  # third delta is an outlier -> clipped to 3x running average
    for i in range(3):
        comp = DeviceCompressor(L, dev, cfg)
        d = torch.zeros(L.total, device=dev)
        for e in L.entries:
            d[e.offset:e.offset + e.numel] = torch.randn(e.numel, device=dev) * 1e-3 * scales_norm[i]
        comp.snap.copy_(theta)
        comp.begin(theta - d)
        comp.finish()
        torch.cuda.synchronize()
        K = comp.read_stats()["num_params_kept"]
        p = comp.payload
        keep.append(comp)
        w = 1000.0 * (i + 1) * 0.9 ** i
        weights.append(w)
        contribs.append(Contribution(idx_ptr=p.idx.data_ptr(), q_ptr=p.q.data_ptr(), val_ptr=p.val.data_ptr(),
                                     win_ptr=p.win.data_ptr(),
                                     scales_ptr=p.scales.data_ptr(), count=K, block=256, dense=False, weight=w,
                                     wire_bytes=p.wire_bytes(K)))
        deq = dequantize_int8(p.q[:K].cpu(), p.scales[:(K + 255) // 256].cpu(), 256)
        dense = torch.zeros(L.total)
        dense[p.idx[:K].long().cpu()] = deq
        dense_deltas.append({e.name: dense[e.offset:e.offset + e.numel] for e in L.entries})
    own = torch.zeros(L.total, device=dev) if in_place else None
    merger = DeviceMerger(L.total, dev, theta, momentum=momentum, theta_buffer=own)
    s32 = torch.zeros(L.total, device=dev)
    dests = [s32.data_ptr()] + ([own.data_ptr()] if in_place else [])  # the own slot is skipped by the kernel
    torch.cuda.synchronize()  # the merger's stream does not wait for the default stream's fills
    info = merger.merge(contribs, 1.0, stage32=dests)
    torch.cuda.synchronize()
    ck = {e.name: theta[e.offset:e.offset + e.numel].cpu() for e in L.entries}
    new, _, rinfo = merge_reference(ck, dense_deltas, weights, outer_lr=1.0, outer_momentum=momentum)
    got = merger.theta.cpu()
    for e in L.entries:
        assert torch.allclose(got[e.offset:e.offset + e.numel], new[e.name], atol=1e-7, rtol=1e-5), e.name
    assert info["accepted"] == 3
    assert info["per_delta_norms"][2] < info["per_delta_norms"][0] * 3.0001 * 2
    assert torch.equal(s32, merger.theta)
    if in_place:
        assert merger.theta.data_ptr() == own.data_ptr()
    if merger.acc is not None:
        assert float(merger.acc.abs().max()) == 0.0


@pytest.mark.parametrize("merge_sms", [0, 16])
def test_inbox_single_gpu_protocol(merge_sms):
    """One node + coordinator on one GPU: pushes, merges, version swaps, loss decreases; the merge on a
    priority stream over the whole GPU, or in a 16-SM green-context partition."""
    from distrain_b200.config import bench_config
    from distrain_b200.parallel.node import InBoxNode
    run = bench_config("micro")
    run.merge_sms = merge_sms
    run.model.vocab_size = 512
    run.push_every = 6
    run.optim.lr = 3e-3
    node = InBoxNode(run, rank=0, world=1, device=torch.device("cuda"), enable_push=True)
    g = torch.Generator().manual_seed(0)
    batch = torch.randint(0, 512, (run.micro_batch, run.seq_len), generator=g, dtype=torch.int32).cuda()
    losses = []
    for i in range(60):
        node.train_step_device(batch)
        losses.append(node.engine.loss[0].item())
    import time
    time.sleep(0.5)
    coord = node.sync.coord
    assert coord.error is None, repr(coord.error)
    assert len(coord.merges) >= 3, (coord.merges, node.sync.seq, coord.next_seq, node.sync.bus.d)
    assert node.sync.version >= 2
    m = coord.merges[-1]
    assert m["accepted"] == 1 and m["pulled_bytes"] > 0
    assert losses[-1] < losses[0]
    node.close()


@pytest.mark.parametrize("rebase,fold", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_swap_in_kernel(rebase, fold):
    """Checkpoint swap against its fp32 definition: replace (master = snap = staged) or rebase
    (master = staged + master - snap, snap = staged), optionally folding the error-feedback residual into
    the weights (master -= ef, ef = 0); bf16 copy of the new master."""
    from distrain_b200.ops._lib import lib, register, check, c_void, c_ll, c_int, stream_ptr
    register("dt_swap_in", [c_void, c_void, c_void, c_void, c_void, c_void, c_ll, c_int, c_void])
    n = 1 << 20
    g = torch.Generator(device="cuda").manual_seed(5)
    s32 = torch.randn(n, device="cuda", generator=g)
    s16 = s32.bfloat16()
    master = torch.randn(n, device="cuda", generator=g)
    snap = master - 1e-3 * torch.randn(n, device="cuda", generator=g)
    ef = 1e-3 * torch.randn(n, device="cuda", generator=g)
    want = s32.double()
    if rebase:
        want = want + (master.double() - snap.double())
    if fold:
        want = want - ef.double()
    want = want.float()
    p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    check(lib().dt_swap_in(s32.data_ptr(), s16.data_ptr(), master.data_ptr(), p16.data_ptr(), snap.data_ptr(),
                           ef.data_ptr() if fold else None, n, rebase,
                           stream_ptr(torch.cuda.current_stream())), "dt_swap_in")
    torch.cuda.synchronize()
    assert torch.allclose(master, want, atol=1e-6, rtol=1e-6)
    assert torch.equal(snap, s32)
    assert torch.equal(p16, master.bfloat16())
    if fold:
        assert float(ef.abs().max()) == 0.0


@pytest.mark.parametrize("swap_mode,ef_on_swap", [("push_partial", "keep"), ("rebase", "keep"),
                                                  ("push_partial", "reset"), ("rebase", "fold")])
def test_inbox_swap_policies(swap_mode, ef_on_swap):
    """The swap policies run the protocol end to end on one GPU (rebase keeps whole rounds: every push
    after the first covers push_every steps)."""
    from distrain_b200.config import bench_config
    from distrain_b200.parallel.node import InBoxNode
    run = bench_config("micro")
    run.model.vocab_size = 512
    run.push_every = 6
    run.optim.lr = 3e-3
    run.swap_mode, run.ef_on_swap = swap_mode, ef_on_swap
    node = InBoxNode(run, rank=0, world=1, device=torch.device("cuda"), enable_push=True)
    g = torch.Generator().manual_seed(0)
    batch = torch.randint(0, 512, (run.micro_batch, run.seq_len), generator=g, dtype=torch.int32).cuda()
    losses = []
    for i in range(60):
        node.train_step_device(batch)
        losses.append(node.engine.loss[0].item())
    import json
    import time
    time.sleep(0.5)
    coord = node.sync.coord
    assert coord.error is None, repr(coord.error)
    assert len(coord.merges) >= 3 and node.sync.version >= 2
    assert losses[-1] < losses[0]
    if swap_mode == "rebase":
        steps = [json.loads(node.sync.bus.get(f"push/0/{s}"))["inner_steps"] for s in range(1, node.sync.seq + 1)]
        assert all(s >= run.push_every for s in steps), steps
    node.close()


def test_distributed_merger_single_node_matches_reference():
    """The distributed merger with one node (its slice is the whole range) against the fp32 reference."""
    from distrain_b200.config import CompressionConfig
    from distrain_b200.parallel.compression import DeviceCompressor, dequantize_int8
    from distrain_b200.parallel.merge import DistributedMerger, Contribution, merge_reference
    L = _layout()
    dev = torch.device("cuda")
    torch.manual_seed(2)
    theta0 = torch.randn(L.total, device=dev) * 0.02
    cfg = CompressionConfig(top_k_fraction=0.2, quantize_int8=True, int8_block=256)
    contribs, dense_deltas, weights, keep, stats = [], [], [], [], []
    for i, sc in enumerate([1.0, 4.0]):
        comp = DeviceCompressor(L, dev, cfg)
        d = torch.randn(L.total, device=dev) * 1e-3 * sc
        comp.snap.copy_(theta0)
        comp.begin(theta0 - d)
        comp.finish()
        torch.cuda.synchronize()
        st = comp.read_stats()
        K = st["num_params_kept"]
        stats.append(st["wire"])
        p = comp.payload
        keep.append(comp)
        w = 1000.0 / (i + 1)
        weights.append(w)
        contribs.append(Contribution(idx_ptr=p.idx.data_ptr(), q_ptr=p.q.data_ptr(), val_ptr=p.val.data_ptr(),
                                     scales_ptr=p.scales.data_ptr(), win_ptr=p.win.data_ptr(), count=K, block=256,
                                     dense=False, weight=w))
        deq = dequantize_int8(p.q[:K].cpu(), p.scales[:(K + 255) // 256].cpu(), 256)
        dense = torch.zeros(L.total)
        dense[p.global_indices(K).cpu()] = deq
        dense_deltas.append({e.name: dense[e.offset:e.offset + e.numel] for e in L.entries})
    theta = theta0.clone()
    ctl = torch.zeros(DistributedMerger.CTL_BYTES, dtype=torch.uint8, device=dev)
    dm = DistributedMerger(0, 1, L.total, dev, theta, [theta.data_ptr()], 0, ctl, [ctl.data_ptr()])
    torch.cuda.synchronize()
    ck = {e.name: theta0[e.offset:e.offset + e.numel].cpu() for e in L.entries}
    for att in (1, 2):
        info = dm.run_local(contribs, stats, 1.0, att)
        ck, _, rinfo = merge_reference(ck, dense_deltas, weights, outer_lr=1.0, outer_momentum=0.0)
        got = theta.cpu()
        for e in L.entries:
            assert torch.allclose(got[e.offset:e.offset + e.numel], ck[e.name], atol=1e-7, rtol=1e-5), (att, e.name)
        assert info["accepted"] == 2


@pytest.mark.parametrize("fused", [False, True])
def test_distributed_merger_slices_on_one_gpu(fused):
    """Three slices of one checkpoint merged one after another on one GPU (a three-node merge whose nodes
    share one staging slot), two quantised sparse members and one raw dense member, against the fp32
    reference: every slice boundary and (fused path) every tile boundary is crossed. The completion
    counter is read only after all three slices finished."""
    from distrain_b200.config import CompressionConfig
    from distrain_b200.parallel.compression import DeviceCompressor, dequantize_int8
    from distrain_b200.parallel.merge import DeviceMerger, DistributedMerger, Contribution, merge_reference
    L = _layout()
    dev = torch.device("cuda")
    torch.manual_seed(5)
    theta0 = torch.randn(L.total, device=dev) * 0.02
    cfg = CompressionConfig(top_k_fraction=0.3, quantize_int8=True, int8_block=256)
    contribs, dense_deltas, weights, keep, stats = [], [], [], [], []
    for i, sc in enumerate([1.0, 2.0, 1.5]):
        comp = DeviceCompressor(L, dev, cfg)
        d = torch.randn(L.total, device=dev) * 1e-3 * sc
        comp.snap.copy_(theta0)
        comp.begin(theta0 - d)
        w = 1000.0 / (i + 1)
        weights.append(w)
        dense = torch.zeros(L.total)
        if i < 2:
            comp.finish()
            torch.cuda.synchronize()
            st = comp.read_stats()
            K = st["num_params_kept"]
            p = comp.payload
            contribs.append(Contribution(idx_ptr=p.idx.data_ptr(), q_ptr=p.q.data_ptr(), val_ptr=p.val.data_ptr(),
                                         scales_ptr=p.scales.data_ptr(), win_ptr=p.win.data_ptr(), count=K,
                                         block=256, dense=False, weight=w))
            dense[p.global_indices(K).cpu()] = dequantize_int8(p.q[:K].cpu(), p.scales[:(K + 255) // 256].cpu(), 256)
        else:
            out = torch.empty(L.total, device=dev)
            comp.finish_raw(out)
            torch.cuda.synchronize()
            st = comp.read_stats(raw=True)
            keep.append(out)
            contribs.append(Contribution(idx_ptr=0, q_ptr=0, val_ptr=out.data_ptr(), scales_ptr=0, win_ptr=0,
                                         count=L.total, block=1, dense=True, weight=w))
            dense = out.cpu()
        stats.append(st["wire"])
        keep.append(comp)
        dense_deltas.append({e.name: dense[e.offset:e.offset + e.numel] for e in L.entries})
    theta = theta0.clone()
    W = 3
    ctls = [torch.zeros(DistributedMerger.CTL_BYTES, dtype=torch.uint8, device=dev) for _ in range(W)]
    dms = [DistributedMerger(r, W, L.total, dev, theta, [theta.data_ptr()] * W, 0, ctls[r],
                             [c.data_ptr() for c in ctls], fused=fused) for r in range(W)]
    assert dms[0].b - dms[0].a > 4 * dms[0].tile  # every slice spans several tiles
    torch.cuda.synchronize()
    ck = {e.name: theta0[e.offset:e.offset + e.numel].cpu() for e in L.entries}
    for att in (1, 2):
        coefs, info = DeviceMerger.plan(contribs, stats)
        for dm in dms:
            dm.apply(contribs, coefs, 1.0)
            dm.check()
        dms[0].finish(att)
        ck, _, rinfo = merge_reference(ck, dense_deltas, weights, outer_lr=1.0, outer_momentum=0.0)
        got = theta.cpu()
        for e in L.entries:
            assert torch.allclose(got[e.offset:e.offset + e.numel], ck[e.name], atol=1e-7, rtol=1e-5), (att, e.name)
        assert info["accepted"] == 3


def test_raw_push_kernel():
    """Raw push: the dense delta + error feedback leaves as fp32, error feedback cleared, statistics of
    the whole delta."""
    from distrain_b200.config import CompressionConfig
    from distrain_b200.parallel.compression import DeviceCompressor
    L = _layout()
    dev = torch.device("cuda")
    comp = DeviceCompressor(L, dev, CompressionConfig(top_k_fraction=0.1))
    master = torch.randn(L.total, device=dev) * 0.02
    d = torch.randn(L.total, device=dev) * 1e-3
    e0 = torch.randn(L.total, device=dev) * 1e-4
    comp.snap.copy_(master + d)
    comp.ef.copy_(e0)
    out = torch.empty(L.total, device=dev)
    comp.begin(master)
    comp.finish_raw(out)
    torch.cuda.synchronize()
    want = torch.zeros(L.total, device=dev)
    for e in L.entries:
        sl = slice(e.offset, e.offset + e.numel)
        want[sl] = (master + d)[sl] - master[sl] + e0[sl]
    for e in L.entries:
        sl = slice(e.offset, e.offset + e.numel)
        torch.testing.assert_close(out[sl], want[sl], rtol=0, atol=1e-7)
    assert float(comp.ef.abs().max()) == 0.0
    st = comp.read_stats(raw=True)
    assert st["num_params_kept"] == L.total
    assert abs(st["dense_norm"] - float(want.double().norm())) < 1e-6 * st["dense_norm"]
    assert st["sparse_norm"] == st["dense_norm"]


def test_inbox_bandwidth_adaptive_protocol():
    """Bandwidth-adaptive pushes on one GPU: the first push is a loss-based top-k (no bandwidth measured
    yet), later pushes are raw once the merge has measured the pull rate; merges apply them."""
    import json
    import time
    from distrain_b200.config import bench_config
    from distrain_b200.parallel.node import InBoxNode
    run = bench_config("micro")
    run.model.vocab_size = 512
    run.push_every = 6
    run.optim.lr = 3e-3
    run.bandwidth_adaptive = True
    node = InBoxNode(run, rank=0, world=1, device=torch.device("cuda"), enable_push=True)
    g = torch.Generator().manual_seed(0)
    batch = torch.randint(0, 512, (run.micro_batch, run.seq_len), generator=g, dtype=torch.int32).cuda()
    losses = []
    for i in range(60):
        node.train_step_device(batch)
        losses.append(node.engine.loss[0].item())
    time.sleep(0.5)
    coord = node.sync.coord
    assert coord.error is None, repr(coord.error)
    assert not coord.failed, coord.failed
    bodies = [json.loads(node.sync.bus.get(f"push/0/{s}")) for s in range(1, node.sync.seq + 1)]
    assert bodies[0]["_dense"] == 0 and any(b["_dense"] == 1 for b in bodies[1:]), [b["_dense"] for b in bodies]
    assert len(coord.merges) >= 3 and losses[-1] < losses[0]
    node.close()


def test_inbox_checkpoint_store_and_resume(tmp_path):
    """The one-GPU protocol stores every merged version in the reference layout; a restarted node resumes
    from the newest one (weights, bf16 copy, version)."""
    import time
    from distrain_b200.config import bench_config
    from distrain_b200.parallel.node import InBoxNode
    from distrain_b200.parallel.inbox_ckpt import latest_version, resume_flat
    from distrain_b200.utils.storage import FsStore
    run = bench_config("micro")
    run.model.vocab_size = 512
    run.push_every = 6
    run.optim.lr = 3e-3
    run.checkpoint_store = str(tmp_path)
    run.checkpoint_every = 1
    run.keep_versions = 3
    node = InBoxNode(run, rank=0, world=1, device=torch.device("cuda"), enable_push=True)
    g = torch.Generator().manual_seed(0)
    batch = torch.randint(0, 512, (run.micro_batch, run.seq_len), generator=g, dtype=torch.int32).cuda()
    for i in range(40):
        node.train_step_device(batch)
    time.sleep(0.5)
    node.close()  # joins the coordinator (a merge in flight completes) and flushes the checkpoint writer
    merged = node.sync.coord.version
    store = FsStore(str(tmp_path))
    v = latest_version(store)
    assert v is not None and v == merged >= 1  # every merged version is stored (checkpoint_every=1)
    flat = resume_flat(store, node.engine.layout, v)
    assert torch.isfinite(flat).all()
    del node
    torch.cuda.empty_cache()
    run.resume = True
    node2 = InBoxNode(run, rank=0, world=1, device=torch.device("cuda"), enable_push=True)
    assert node2.sync.version == v and node2.sync.coord.version == v
    L = node2.engine.layout
    for e in L.entries:
        sl = slice(e.offset, e.offset + e.numel)
        assert torch.equal(node2.engine.master[sl].cpu(), flat[sl]), e.name
    assert torch.equal(node2.engine.p16, node2.engine.master.bfloat16())
    node2.train_step_device(batch)
    node2.close()
