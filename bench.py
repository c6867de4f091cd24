"""Headline benchmark: aggregate training tokens/s of asynchronous data-parallel nodes, one per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config tiny] [--impl dt|reference]

For N > 1 launch with ``python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ...``.
Each rank is one Distrain node: the tiny preset (hidden 768, 12 layers, 12 heads / 4 KV heads, SwiGLU
2048, vocab 32768) at seq 1024 x micro-batch 32, bf16 compute with fp32 master weights and AdamW
state, synthetic uniform-random tokens from per-rank seeds, N(0, 0.02) init. Every ``push_every``
steps each node compresses its delta (top-k 10% + per-block INT8 with error feedback) and the
coordinator merges the pushed deltas with 0.9^staleness x tokens weights and applies them unscaled.

Timing: W untimed warm-up steps, then exactly K steps bracketed by barrier + device synchronisation,
timed with CUDA events on the training stream; the reported time is the max over ranks. A training
step's working set (~12 GB of activations and state) is far larger than the 126 MB L2, so no L2
flush is inserted. ``e2e`` repeats the K steps through the public node API with a pinned-host H2D
copy of every step's tokens and a D2H read of every step's loss.

Protocol inside the timed steps: before each timed region every node's round counter is phased so its
push falls after step K/2 of the region (``InBoxNode.phase_push``); the compression, the coordinator's
merge and broadcast, and the nodes' checkpoint swap then run during the remaining timed steps. The
line's ``merge`` block counts the pushes and swaps that happened inside each region (the minimum over
ranks), so one push per K steps is charged to the measured rate - more than the configured one per
``push_every`` steps whenever K < push_every.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def _parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="tiny")
    ap.add_argument("--impl", default="dt", choices=["dt", "reference"])
    ap.add_argument("--push-every", type=int, default=None)
    ap.add_argument("--grad-accum", type=int, default=None, help="micro-batches per optimizer step")
    ap.add_argument("--merge-sms", type=int, default=None,
                    help="SMs of the green-context partition the merge kernels run in (0 = priority stream)")
    ap.add_argument("--tp", type=int, default=None, help="tensor-parallel size per node (default: the preset's)")
    ap.add_argument("--clocks-csv", default=None,
                    help="keep the nvidia-smi clock samples of the timed region in this CSV (default: a temp file)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-push", action="store_true", help="train only (no compression / merge)")
    ap.add_argument("--tp-mode", default="fused", choices=["fused", "nccl"],
                    help="tensor-parallel partial-sum exchange: fused GEMM-epilogue peer stores, or NCCL all-reduce")
    ap.add_argument("--sync", default="inbox", choices=["inbox", "nccl"],
                    help="inbox: compressed deltas, peer-pull merge kernel, NVLS broadcast (the product); "
                         "nccl: comparison arm, dense fp32 delta all-reduce every push")
    return ap.parse_args()


def reference_unavailable(args):
    line = {"impl": "reference",
            "unavailable": "the reference (frane/distrain) is a Rust/Burn workspace and this image has no cargo/rustc "
                           "toolchain, so it cannot be built or run offline"}
    print(json.dumps(line), flush=True)


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region (rank 0, all visible GPUs)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, path):
        self.path = path
        self.proc = None

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def _merge_list(node, nccl_arm):
    """Merges completed so far (rank 0's coordinator; the NCCL arm's all-reduce steps); [] elsewhere."""
    if node.sync is None:
        return []
    if nccl_arm:
        return list(node.sync.merges)
    return list(node.sync.coord.merges) if node.sync.coord is not None else []


def main():
    args = _parse()
    if args.impl == "reference":
        reference_unavailable(args)
        return 0
    import torch
    import torch.distributed as dist
    from distrain_b200.config import bench_config
    from distrain_b200.parallel.node import InBoxNode
    from distrain_b200 import ops
    from distrain_b200.utils.tracing import nvtx, setup_logging
    from distrain_b200.roofline import step_roofline
    setup_logging()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world > 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        # NCCL's communicator set-up lines (ranks, devices, transports) stay on, on stderr, so the ranks and
        # GPUs of the run can be checked; stdout stays the one JSON line
        os.environ["NCCL_DEBUG"] = "INFO"
        os.environ["NCCL_DEBUG_SUBSYS"] = os.environ.get("NCCL_DEBUG_SUBSYS") or "INIT"
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=300))
    run = bench_config(args.config)
    if args.push_every:
        run.push_every = args.push_every
    if args.grad_accum:
        run.grad_accum_steps = max(args.grad_accum, 1)
    if args.merge_sms is not None:
        run.merge_sms = max(args.merge_sms, 0)
    if args.tp:
        run.tp = args.tp
    nccl_arm = args.sync == "nccl" and not args.no_push
    # tensor parallelism: node k = ranks [k*tp, (k+1)*tp); its shards are averaged across nodes by the
    # groups of ranks that hold the same shard
    tp_size = run.tp if (run.tp > 1 and world % run.tp == 0) else 1
    tp, dp_group = None, None
    if tp_size > 1:
        from distrain_b200.parallel.tensor_parallel import TensorParallel
        nodes = world // tp_size
        tp_groups = [dist.new_group([k * tp_size + i for i in range(tp_size)]) for k in range(nodes)]
        dp_groups = [dist.new_group([k * tp_size + i for k in range(nodes)]) for i in range(tp_size)]
        tp = TensorParallel(tp_groups[rank // tp_size], rank % tp_size, tp_size, mode=args.tp_mode,
                            rows=run.micro_batch * (run.seq_len - 1), hidden=run.model.hidden_dim, device=dev)
        dp_group = dp_groups[rank % tp_size]
    node_rank, n_nodes = rank // tp_size, world // tp_size
    if rank == 0:
        from distrain_b200.memory import check_fits
        fits, est = check_fits(run, torch.cuda.get_device_properties(dev).total_memory, n_nodes,
                               protocol=not args.no_push)
        if not fits:
            print(f"warning: {run.name} needs ~{est['total'] / 1e9:.0f} GB per rank (engine {est['engine'] / 1e9:.0f}, "
                  f"activations {est['activations'] / 1e9:.0f}, protocol {est['protocol'] / 1e9:.0f}); this GPU has "
                  f"{torch.cuda.get_device_properties(dev).total_memory / 1e9:.0f} GB - use tensor parallelism "
                  f"(--tp) or fewer payload slots", file=sys.stderr)
    # with tensor parallelism every rank runs the protocol for its shard over its dp group
    node = InBoxNode(run, rank=node_rank, world=n_nodes, device=dev,
                     enable_push=not args.no_push and not nccl_arm, tp=tp,
                     shard=rank % tp_size, n_shards=tp_size, dp_group=dp_group)
    if nccl_arm:
        from distrain_b200.parallel.nccl_baseline import NcclDenseSync
        node.sync = NcclDenseSync(node, run, node_rank, n_nodes, dev, group=dp_group)
    B, S, A = run.micro_batch, run.seq_len, run.grad_accum_steps

    # synthetic uniform-random tokens, per-node seed (the ranks of one tensor-parallel node share them)
    g = torch.Generator().manual_seed(1000 + node_rank)
    ring = [torch.randint(0, run.model.vocab_size, (A * B, S), generator=g, dtype=torch.int32).pin_memory()
            for _ in range(4)]
    dev_batches = [r.to(dev) for r in ring]

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up (also captures the CUDA graph). With 3+ warm-up steps a push falls after the first one, so the
    # first compression, merge and broadcast (and their one-time costs: lazy kernel loading, allocator
    # growth) complete before the timed regions; the merges of the timed regions are reported apart.
    warm_push = node.sync is not None and args.warmup >= 3
    if warm_push:
        node.phase_push(1)
    with nvtx("warmup"):
        for i in range(args.warmup):
            node.train_step_device(dev_batches[i % 4])
    torch.cuda.synchronize()
    if warm_push and rank == 0:
        t_w = time.time()
        while not _merge_list(node, nccl_arm) and time.time() - t_w < 120:
            time.sleep(0.005)
    barrier()
    n_warm_merges = len(_merge_list(node, nccl_arm))

    clocks = None
    if rank == 0:
        if args.clocks_csv:
            path = args.clocks_csv
            os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        else:
            import tempfile
            fd, path = tempfile.mkstemp(prefix="dt_clocks_", suffix=".csv")
            os.close(fd)
        clocks = ClockSampler(path)
        clocks.start()
        time.sleep(0.5)

    def protocol_marks():
        s = node.sync
        return (s.seq, s.version) if s is not None else (0, 0)

    def phase():
        if node.sync is not None:
            node.phase_push(max(args.steps // 2, 1))

    ops._lib.LAUNCHES[0] = 0
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    phase()
    marks0 = protocol_marks()
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    with nvtx("timed"):
        for i in range(args.steps):
            node.train_step_device(dev_batches[i % 4])
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    launches = ops._lib.LAUNCHES[0]
    ms = e0.elapsed_time(e1)
    marks_dev_end = marks1 = protocol_marks()

    e2e_ms = None
    marks2 = marks1
    if not args.no_e2e:
        phase()
        marks1 = protocol_marks()
        barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        with nvtx("timed_e2e"):
            losses = node.train_steps_e2e(ring, args.steps)
        f1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = f0.elapsed_time(f1)
        marks2 = protocol_marks()
    clk = clocks.stop() if clocks else None

    free_b, total_b = torch.cuda.mem_get_info(dev)
    t = torch.tensor([ms, e2e_ms or 0.0, float(launches), float(total_b - free_b)], device=dev)
    # pushes / swaps inside the device-timed and the e2e regions, negated so that the MAX reduction
    # yields the minimum over ranks
    t = torch.cat([t, -torch.tensor([marks_t[0] - marks_s[0] for marks_s, marks_t in
                                     ((marks0, marks_dev_end), (marks1, marks2))] +
                                    [marks_t[1] - marks_s[1] for marks_s, marks_t in
                                     ((marks0, marks_dev_end), (marks1, marks2))], dtype=torch.float32, device=dev)])
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms_max, launches, mem_used = t[0].item(), t[1].item(), int(t[2].item()), t[3].item()
    pushes_dev, pushes_e2e, swaps_dev, swaps_e2e = (int(-x) for x in t[4:8].tolist())
    merges = _merge_list(node, nccl_arm)[n_warm_merges:]
    versions = node.sync.version if node.sync is not None else 0
    node.close()
    tokens_per_step = A * B * S
    value = tokens_per_step * n_nodes * args.steps / (ms / 1e3)
    if rank == 0:
        out = {
            "metric": "train tokens/sec (aggregate over GPUs, max-over-ranks time)",
            "value": round(value, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (uniform-random token ids, per-rank seeds; random-init N(0,0.02) weights)",
            "config": {"model": f"{run.name} preset ({run.model.param_count()/1e6:.1f}M params)",
                       "global_batch": A * B * n_nodes, "seq_len": S,
                       "micro_batch": B, "grad_accum_steps": A,
                       "merge_partition": (f"green context of {run.merge_sms}+ SMs" if run.merge_sms > 0
                                           else "top-priority stream, whole GPU"),
                       "parallelism": ((f"tp{tp_size} ({args.tp_mode} exchange) x " if tp_size > 1 else "") +
                                       (f"sync-dp{n_nodes} (NCCL all-reduce of dense fp32 deltas every push)"
                                        if nccl_arm else f"async-dp{n_nodes} (1 node per GPU)")),
                       "activation_checkpointing": run.activation_checkpointing,
                       "push_every": run.push_every if not args.no_push else None,
                       "compression": ("none (dense fp32 delta)" if nccl_arm else
                                       f"top-k {run.compression.top_k_fraction:.0%} + INT8 block "
                                       f"{run.compression.int8_block} + error feedback"),
                       "l2": (f"per-step working set >= {node.engine.layout.total * 18 / 1e9:.1f} GB (weights, "
                              "gradients, AdamW state) >> 126 MB L2; no flush"),
                       "device_memory_used_gb_max": round(mem_used / 1e9, 1)},
            "gpu_launches": launches,
            "clocks": clk,
            # model FLOPs (6N + causal attention [+ recompute]) per GPU against the measured bf16 peaks
            "roofline": step_roofline(run.model, S, value, world, run.activation_checkpointing),
        }
        if node.sync is not None and not merges:
            out["merge"] = {"count": 0, "pushes_in_timed_steps": pushes_dev, "swaps_in_timed_steps": swaps_dev,
                            "note": "no merge completed before the end of the run"}
        if merges:
            dev_ms = sorted(m["device_ms"] for m in merges)
            out["merge"] = {"count": len(merges), "node_version": versions,
                            "warmup_merges": n_warm_merges,
                            "ms_median": round(dev_ms[(len(dev_ms) - 1) // 2], 3),
                            "device_ms_each": [round(m["device_ms"], 3) for m in merges],
                            "wall_ms_each": [round(m.get("wall_ms", 0.0), 3) for m in merges],
                            "timing": ("CUDA events on rank 0's merge stream while the nodes train, host planning "
                                       "and control-bus round trips between its kernels included") if not nccl_arm else
                                      "CUDA events around the NCCL all-reduce + apply on the training stream",
                            "pushes_in_timed_steps": pushes_dev, "swaps_in_timed_steps": swaps_dev,
                            "pushes_in_e2e_steps": pushes_e2e if e2e_ms is not None else None,
                            "swaps_in_e2e_steps": swaps_e2e if e2e_ms is not None else None,
                            "push_phase": f"push after step {max(args.steps // 2, 1)} of each timed region",
                            "contributions_last": merges[-1]["n_contrib"],
                            "pulled_bytes_last": merges[-1]["pulled_bytes"],
                            "broadcast_bytes_last": merges[-1]["broadcast_bytes"],
                            "multicast": merges[-1]["multicast"],
                            "phases_ms_last": merges[-1].get("phases_ms")}
            if nccl_arm:
                out["merge"]["allreduce_bytes"] = merges[-1]["allreduce_bytes"]
        if e2e_ms is not None:
            out["e2e"] = {"value": round(tokens_per_step * n_nodes * args.steps / (e2e_ms_max / 1e3), 1),
                          "unit": "tokens/s", "h2d_bytes_per_step": A * B * S * 4, "d2h_bytes_per_step": 4}
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
