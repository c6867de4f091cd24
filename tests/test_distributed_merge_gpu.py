"""Distributed merge (every node merges one slice of the checkpoint) against the fp32 reference merge.

Two spawned ranks on two GPUs each compress their own delta into a symmetric payload buffer and report
its statistics; both plan from them, merge their slice and broadcast it, twice; after each attempt both
ranks' staging slots must hold the reference merge of both dequantised deltas (staleness-style weights,
3x-average norm clip) applied to the previous checkpoint. Skipped on a one-GPU box (the one-GPU case is
in test_compress_merge_gpu.py)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, out_dir, merge_sms=0):
    import datetime
    import torch.distributed as dist
    from distrain_b200.config import CompressionConfig, preset
    from distrain_b200.models.params import ParamLayout
    from distrain_b200.parallel.compression import DeviceCompressor, DevicePayload
    from distrain_b200.parallel.inbox import _symm_alloc
    from distrain_b200.parallel.merge import Contribution, DeviceMerger, DistributedMerger
    from distrain_b200.parallel.partition import merge_stream
    from distrain_b200 import ops
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    W = 2
    L = ParamLayout(preset("micro"))
    n = L.total
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    theta0 = torch.randn(n, device=dev, generator=torch.Generator(device="cuda").manual_seed(7)) * 0.02
    scale = [1.0, 5.0][rank]  # rank 1's delta is an outlier: clipped to 3x rank 0's norm
    delta = torch.randn(n, device=dev, generator=g) * 1e-3 * scale
    cfg = CompressionConfig(top_k_fraction=0.2, quantize_int8=True, int8_block=256)
    cap = DeviceCompressor.capacity_for(L, 0.2)
    pay_buf, pay_ptrs, _, _h1 = _symm_alloc((DevicePayload.nbytes(cap, 256) + 4095) // 4096 * 4096, dev, W)
    payload = DevicePayload(pay_buf[:DevicePayload.nbytes(cap, 256)], cap, 256)
    comp = DeviceCompressor(L, dev, cfg, payload=payload)
    comp.snap.copy_(theta0)
    comp.begin(theta0 - delta)
    comp.finish()
    torch.cuda.synchronize()
    st = comp.read_stats()
    K = st["num_params_kept"]
    cnt = torch.tensor([K] + st["wire"], device=dev, dtype=torch.float64)
    got = [torch.zeros_like(cnt) for _ in range(W)]
    dist.all_gather(got, cnt)
    counts = [int(g[0]) for g in got]
    stats = [g[1:].tolist() for g in got]
    stage_buf, stage_ptrs, stage_mc, _h2 = _symm_alloc((n * 4 + 4095) // 4096 * 4096, dev, W)
    theta = stage_buf[:n * 4].view(torch.float32)
    theta.copy_(theta0)
    ctl, ctl_ptrs, _, _h3 = _symm_alloc(DistributedMerger.CTL_BYTES, dev, W)
    dm = DistributedMerger(rank, W, n, dev, theta, stage_ptrs, stage_mc, ctl, ctl_ptrs,
                           stream=merge_stream(dev, merge_sms))
    base = pay_buf.data_ptr()
    weights = [1000.0, 800.0 * 0.9]
    contribs = []
    for r in range(W):
        off = lambda t, r=r: t.data_ptr() - base + pay_ptrs[r]
        contribs.append(Contribution(idx_ptr=off(payload.idx), q_ptr=off(payload.q), val_ptr=off(payload.val),
                                     scales_ptr=off(payload.scales), win_ptr=off(payload.win), count=counts[r],
                                     block=256, dense=False, weight=weights[r]))
    torch.cuda.synchronize()
    dist.barrier()
    slots, infos = [], []
    for att in (1, 2):
        coefs, info = DeviceMerger.plan(contribs, stats)
        infos.append(info)
        dist.barrier()
        dm.apply(contribs, coefs, 1.0)
        dm.check()
        dist.barrier()
        if rank == 0:
            dm.finish(att)
        dist.barrier()
        slots.append(theta.cpu().clone())
        if att == 1:
            diag = {"ranges": ctl[dm.OFF_RANGES:dm.OFF_RANGES + 16 * W].view(torch.int64).cpu().clone(),
                    "coefs": ctl[dm.OFF_COEF:dm.OFF_COEF + 4 * W].view(torch.float32).cpu().clone(),
                    "stats": torch.tensor(stats), "a": dm.a, "b": dm.b, "mc": int(stage_mc or 0)}
    gi = payload.global_indices(K).cpu()
    deq = (payload.q[:K].float() * payload.scales[torch.arange(K, device=dev) // 256]).cpu()
    torch.save({"slots": slots, "idx": gi, "val": deq, "theta0": theta0.cpu(), "infos": infos, "diag": diag,
                "err": ops.device_error()[0], "weights": weights},
               os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("merge_sms", [0, 16])
def test_distributed_merge_two_gpus(tmp_path, merge_sms):
    """merge_sms 16: every node's slice merge and broadcast run in a 16-SM green-context partition."""
    import torch.multiprocessing as mp
    from distrain_b200.config import preset
    from distrain_b200.models.params import ParamLayout
    from distrain_b200.parallel.merge import merge_reference
    mp.spawn(_rank, args=(_free_port(), str(tmp_path), merge_sms), nprocs=2, join=True)
    res = [torch.load(os.path.join(tmp_path, f"rank{r}.pt")) for r in range(2)]
    assert res[0]["err"] == 0 and res[1]["err"] == 0
    L = ParamLayout(preset("micro"))
    n = L.total
    deltas = []
    for r in range(2):
        d = torch.zeros(n)
        d[res[r]["idx"]] = res[r]["val"]
        deltas.append({e.name: d[e.offset:e.offset + e.numel] for e in L.entries})
    ck = {e.name: res[0]["theta0"][e.offset:e.offset + e.numel] for e in L.entries}
    for att in range(2):
        ck, _, info = merge_reference(ck, deltas, res[0]["weights"], outer_lr=1.0, outer_momentum=0.0)
        want = res[0]["theta0"].clone()  # layout padding between tensors is never touched by a merge
        for e in L.entries:
            want[e.offset:e.offset + e.numel] = ck[e.name]
        for r in range(2):
            got = res[r]["slots"][att]
            if not torch.allclose(got, want, atol=1e-7, rtol=1e-5):
                bad = ((got - want).abs() > 1e-7 + 1e-5 * want.abs()).nonzero().flatten()
                dg = [res[q]["diag"] for q in range(2)]
                # expected ranges from the saved payload indices
                exp = [[int(torch.searchsorted(res[m]["idx"], dg[q]["a"])),
                        int(torch.searchsorted(res[m]["idx"], dg[q]["b"]))] for q in range(2) for m in range(2)]
                t0 = res[0]["theta0"]
                msg = (f"att {att} rank {r}: {bad.numel()} wrong of {n}, first {bad[:5].tolist()} last "
                       f"{bad[-5:].tolist()}; got {got[bad[:3]].tolist()} want {want[bad[:3]].tolist()} theta0 "
                       f"{t0[bad[:3]].tolist()}; ranges {[d['ranges'].tolist() for d in dg]} expected {exp}; "
                       f"coefs {[d['coefs'].tolist() for d in dg]} stats {dg[0]['stats'].tolist()} "
                       f"a/b {[(d['a'], d['b']) for d in dg]} mc {dg[0]['mc']} counts "
                       f"{[res[m]['idx'].numel() for m in range(2)]}")
                raise AssertionError(msg)
        assert torch.equal(res[0]["slots"][att], res[1]["slots"][att])
    assert res[0]["infos"][0]["accepted"] == 2
    assert res[0]["infos"][0]["per_delta_norms"][1] < res[0]["infos"][0]["per_delta_norms"][0] * 3.0001
