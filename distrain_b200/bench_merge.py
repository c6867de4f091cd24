"""Merge microbenchmark on one NVSwitch box: N nodes' compressed deltas -> coordinator merge -> checkpoint
broadcast, against an NCCL all-reduce of the same deltas in dense fp32.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 --master-port P \\
        -m distrain_b200.bench_merge [--models tiny,small] [--topk 0.01,0.1,0.99] [--iters 5] [--warmup 2]

Inputs (per rank seed): a delta of i.i.d. N(0, 1e-4^2) entries over the preset's parameter layout (the
snapshot minus the master weights) and an error-feedback buffer of the same distribution; staleness drawn
uniformly from {0, 1, 2, 3} and token counts uniformly from [1e5, 1e6], giving the merge weights
tokens * 0.9^staleness.

With ``--per-rank K`` every GPU pushes K deltas (K payload buffers, each compressed from its own
snapshot), so the merge has GPUs x K contributors; compress_ms is then one compression.

Per (model, top-k), every iteration:
  1. every rank compresses its delta (+ error feedback) into its symmetric (peer-mapped) payload buffer:
     pass A + radix top-k + ordered compaction + INT8 block 256 (or, for "raw", pass A and the dense fp32
     delta);
  2. the distributed merge: validation, clipping and weights from the statistics every node reports with
     its push, then every rank merges one slice of the flat range - pulls that slice of all N payloads
     over NVLink, adds it into its slice of the checkpoint (its own staging buffer) and writes the slice
     into every rank's staging buffer with NVLS multimem stores, or per-peer stores without a multicast
     object;
  3. for comparison, the single-coordinator merge of the same payloads (rank 0 pulls all of them,
     scatter-adds into its checkpoint and broadcasts the whole checkpoint).
Timed with CUDA events on the launching streams: compress = max over ranks, merge = rank 0, from the
start of its slice to its check that every rank's slice landed (an NCCL barrier, inside the timed
interval, separates the two), total = their sum. Bytes over NVLink: payloads pulled from the N-1 peers plus the
checkpoint stored through the multicast object (each GPU receives it once).
Comparison arm per model: delta = snapshot - master scaled by its merge weight, ncclAllReduce(SUM) of the
n fp32 values, the same apply and bf16 cast on every rank; max over ranks. One JSON line per case on
rank 0.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _max_over_ranks(x: float, dev) -> float:
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_model(name: str, topks, iters: int, warmup: int, rank: int, world: int, dev, per_rank: int = 1):
    from .config import preset, CompressionConfig
    from .models.params import ParamLayout
    from .parallel.compression import DeviceCompressor, DevicePayload
    from .parallel.merge import DeviceMerger, DistributedMerger, Contribution
    from .parallel.inbox import _symm_alloc
    from . import ops

    L = ParamLayout(preset(name))
    n = L.total
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    master = torch.randn(n, device=dev, generator=g) * 0.02
    # per_rank deltas per GPU (contributor j = rank * per_rank + k pushes snaps[k] - master)
    snaps = [master + torch.randn(n, device=dev, generator=g) * 1e-4 for _ in range(per_rank)]
    snap = snaps[0]
    ef0 = torch.randn(n, device=dev, generator=g) * 1e-4
    nc = world * per_rank  # contributors
    hg = torch.Generator().manual_seed(4321)  # same draws on every rank
    stale = torch.randint(0, 4, (nc,), generator=hg).tolist()
    tokens = torch.randint(100_000, 1_000_001, (nc,), generator=hg).tolist()
    weights = [t * 0.9 ** s for t, s in zip(tokens, stale)]
    ks = [k for k in topks if k != "raw"]
    cap_max = DeviceCompressor.capacity_for(L, max(ks)) if ks else 1
    need = DevicePayload.nbytes(cap_max, 256)
    if "raw" in topks:
        need = max(need, 4 * n)
    pay_bytes = (need + 4095) // 4096 * 4096
    pay_buf, pay_ptrs, _, _pay_h = _symm_alloc(pay_bytes * per_rank, dev, world)
    stage_bytes = (n * 4 + 4095) // 4096 * 4096
    stage_buf, stage_ptrs, stage_mc, _stage_h = _symm_alloc(stage_bytes, dev, world)
    p32 = [p for p in stage_ptrs]
    mc32 = stage_mc or 0
    theta = stage_buf[:n * 4].view(torch.float32)
    theta.copy_(snap)
    ctl, ctl_ptrs, _, _ctl_h = _symm_alloc(DistributedMerger.CTL_BYTES, dev, world)
    dm = DistributedMerger(rank, world, n, dev, theta, p32, mc32, ctl, ctl_ptrs)
    single = DeviceMerger(n, dev, None, momentum=0.0, theta_buffer=theta) if rank == 0 else None
    att = 0
    results = []

    def barrier():
        if world > 1:
            dist.barrier()

    for k in topks:
        raw = k == "raw"
        cap = DeviceCompressor.capacity_for(L, 0.01 if raw else k)
        payloads = [DevicePayload(pay_buf[q * pay_bytes:q * pay_bytes + DevicePayload.nbytes(cap, 256)], cap, 256)
                    for q in range(per_rank)]
        comp = DeviceCompressor(L, dev, CompressionConfig(top_k_fraction=0.01 if raw else k, int8_block=256),
                                payload=payloads[0])
        raw_views = [pay_buf[q * pay_bytes:q * pay_bytes + 4 * n].view(torch.float32) for q in range(per_rank)] \
            if raw else None
        t_comp, t_merge, t_single, pulled, infos = [], [], [], 0, None
        for it in range(warmup + iters):
            rows = []
            for q in range(per_rank):
                comp.snap.copy_(snaps[q])
                comp.ef.copy_(ef0)
                torch.cuda.synchronize()
                barrier()
                c0, c1 = _events()
                c0.record()
                comp.begin(master)
                if raw:
                    comp.finish_raw(raw_views[q])
                else:
                    comp.finish(payload=payloads[q])
                c1.record()
                torch.cuda.synchronize()
                if q == 0 and it >= warmup:
                    t_comp.append(c0.elapsed_time(c1))
                kept = n if raw else int(comp.stats_host[comp.nseg * 6].item())
                rows.append([kept] + comp.read_stats(raw=raw)["wire"])
            cnt = torch.tensor(rows, device=dev, dtype=torch.float64)  # [per_rank, 4]
            got = [torch.zeros_like(cnt) for _ in range(world)]
            if world > 1:
                dist.all_gather(got, cnt)
            else:
                got = [cnt]
            counts = [int(g[q, 0].item()) for g in got for q in range(per_rank)]
            stats = [g[q, 1:].tolist() for g in got for q in range(per_rank)]  # what each push reports
            base = pay_buf.data_ptr()
            contribs = []
            for r in range(world):
                for q in range(per_rank):
                    j = r * per_rank + q
                    off = lambda t, r=r: t.data_ptr() - base + pay_ptrs[r]
                    if raw:
                        contribs.append(Contribution(idx_ptr=0, q_ptr=0, val_ptr=off(raw_views[q]), scales_ptr=0,
                                                     count=n, block=0, dense=True, weight=weights[j],
                                                     node_id=f"node-{j:02d}", wire_bytes=4 * n))
                        continue
                    pq = payloads[q]
                    contribs.append(Contribution(idx_ptr=off(pq.idx), q_ptr=off(pq.q), win_ptr=off(pq.win),
                                                 val_ptr=off(pq.val), scales_ptr=off(pq.scales), count=counts[j],
                                                 block=256, dense=False, weight=weights[j], node_id=f"node-{j:02d}",
                                                 wire_bytes=pq.wire_bytes(counts[j])))
            pulled = sum(c.wire_bytes for c in contribs[per_rank:])
            # distributed merge: every rank plans from the reported statistics (the same on every rank),
            # merges its slice and broadcasts it; rank 0 checks that every slice landed
            coefs, infos = DeviceMerger.plan(contribs, stats)
            att += 1
            barrier()
            m0, m1 = _events()
            m0.record(dm.stream)
            dm.apply(contribs, coefs, 1.0)
            dm.check()
            barrier()
            if rank == 0:
                dm.finish(att)
            m1.record(dm.stream)
            dm.stream.synchronize()
            mms = m0.elapsed_time(m1) if rank == 0 else 0.0
            barrier()
            # single-coordinator merge of the same payloads (rank 0 pulls all of them, scatter-adds into its
            # checkpoint and broadcasts the whole of it)
            sms = 0.0
            if rank == 0:
                s0, s1 = _events()
                s0.record(single.stream)
                single.accumulate_apply(contribs, coefs, 1.0, mc32=mc32, stage32=p32)
                s1.record(single.stream)
                single.stream.synchronize()
                sms = s0.elapsed_time(s1)
            barrier()
            if it >= warmup:
                t_merge.append(mms)
                t_single.append(sms)
        cms = _max_over_ranks(sorted(t_comp)[len(t_comp) // 2], dev)
        mms = _max_over_ranks(sorted(t_merge)[len(t_merge) // 2], dev)
        sms = _max_over_ranks(sorted(t_single)[len(t_single) // 2], dev)
        if rank == 0:
            from .roofline import distributed_merge_roofline
            per_member = sum(c.wire_bytes for c in contribs) / len(contribs)
            roof = distributed_merge_roofline(n, per_member * per_rank, world, mms, multicast=bool(mc32))
            results.append({"bench": "compress_merge_broadcast", "model": name, "params": L.num_params(),
                            "merge_roofline": roof, "contributors": nc, "payloads_per_gpu": per_rank,
                            "n_nodes": world, "top_k": k, "compress_ms": round(cms, 3), "merge_ms": round(mms, 3),
                            "total_ms": round(cms + mms, 3), "merge": f"distributed over {world} GPUs",
                            "single_coordinator_merge_ms": round(sms, 3), "accepted": infos["accepted"],
                            "payload_bytes_pulled_nvlink": pulled,
                            "checkpoint_bytes_broadcast": n * 4, "broadcast": "nvls multimem" if mc32 else "per-peer",
                            "staleness": stale, "tokens": tokens,
                            "timing": "CUDA events, median of iters, max over ranks"})
        del comp, payloads
    # comparison arm: dense fp32 all-reduce of the same deltas
    delta = torch.empty_like(master)
    p16t = torch.empty(n, device=dev, dtype=torch.bfloat16)
    theta = torch.empty_like(master)
    ts = []
    for it in range(warmup + iters):
        torch.cuda.synchronize()
        barrier()
        e0, e1 = _events()
        e0.record()
        torch.sub(snap, master, out=delta)
        delta.mul_(weights[rank * per_rank] / sum(weights[::per_rank]))  # the same staleness x tokens weights, then a plain sum
        if world > 1:
            dist.all_reduce(delta, op=dist.ReduceOp.SUM)
        theta.copy_(snap).sub_(delta)
        ops.cast_bf16(theta, p16t)
        e1.record()
        torch.cuda.synchronize()
        if it >= warmup:
            ts.append(e0.elapsed_time(e1))
    ams = _max_over_ranks(sorted(ts)[len(ts) // 2], dev)
    if rank == 0:
        results.append({"bench": "nccl_dense_allreduce", "model": name, "params": L.num_params(), "n_nodes": world,
                        "total_ms": round(ams, 3), "allreduce_bytes_per_rank": n * 4,
                        "bus_bytes_per_rank": int(2 * (world - 1) / world * n * 4),
                        "timing": "CUDA events, median of iters, max over ranks"})
    barrier()
    return results


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--models", default="tiny,small")
    ap.add_argument("--topk", default="0.01,0.1,0.99,raw",
                    help="top-k fractions; 'raw' = the dense fp32 delta (what the bandwidth-adaptive policy sends "
                         "when it fits the upload budget, as it always does over NVLink)")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--per-rank", type=int, default=1,
                    help="payloads pushed per GPU (contributors = GPUs x this): 8 contributors on 4 GPUs with 2")
    a = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=300))
    topks = [x if x == "raw" else float(x) for x in a.topk.split(",")]
    for m in a.models.split(","):
        for r in run_model(m, topks, a.iters, a.warmup, rank, world, dev, max(a.per_rank, 1)):
            print(json.dumps(r), flush=True)
        torch.cuda.empty_cache()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
