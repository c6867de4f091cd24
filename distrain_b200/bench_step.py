"""Per-kernel breakdown of one training step of the engine (CUDA events around every library call).

    python -m distrain_b200.bench_step [--config tiny] [--steps 3] [--warmup 3] [--json]

The step runs eagerly (no CUDA graph) with an event pair around every top-level call into the kernel
library (``ops.*`` and the attention entry points); each call is labelled with its function and the
shapes it was given, and the GEMM-shaped ones with their FLOPs. The sum over calls is compared with
the whole step timed the same way and with the graph-replayed step (the number the benchmark uses):
the difference is launch gaps plus the few torch-side operations of a step. Events between launches
add a little idle time of their own, so read the shares, not the absolute sum.
"""
from __future__ import annotations

import argparse
import collections
import functools
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gemm_label(name, args, kw):
    """(label, flops) of a GEMM-shaped call."""
    if name == "gemm":
        M, N, K = kw["M"], kw["N"], kw["K"]
        tag = "f32acc" if kw.get("epi") == 2 else ("f32" if kw.get("epi") == 1 else "bf16")
        return f"gemm M{M} N{N} K{K} {tag}", 2.0 * M * N * K
    if name in ("linear_fwd", "linear_peer"):
        x, w = args[0], args[1]
        M, K = x.shape
        N = w.shape[0]
        return f"{name} M{M} N{N} K{K}", 2.0 * M * N * K
    if name == "linear_dgrad":
        dy, w = args[0], args[1]
        M, N = dy.shape
        K = w.shape[1]
        return f"{name} M{M} N{K} K{N}", 2.0 * M * N * K
    if name == "linear_wgrad":
        dy, x = args[0], args[1]
        M, N = dy.shape
        K = x.shape[1]
        return f"{name} M{N} N{K} K{M}", 2.0 * M * N * K
    if name.startswith("linear_") or name.startswith("gemm"):
        return name, 0.0
    return None, 0.0


class CallTimer:
    """Wraps the library's entry points with CUDA-event pairs (top-level calls only)."""

    def __init__(self):
        self.records = []
        self.depth = 0
        self.saved = []

    def wrap(self, module, name):
        fn = getattr(module, name)

        @functools.wraps(fn)
        def timed(*args, **kw):
            if self.depth > 0:
                return fn(*args, **kw)
            label, flops = _gemm_label(name, args, kw)
            if label is None:
                label = name
                if name.startswith("attention"):
                    label = f"{name} B{kw.get('B')} T{kw.get('T')} h{kw.get('nh')}/{kw.get('nkv')} d{kw.get('d')}"
                    flops = 4.0 * kw["B"] * kw["nh"] * kw["T"] * kw["T"] * kw["d"] / 2
                    if name == "attention_bwd":
                        flops *= 2.5
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            self.depth += 1
            a.record()
            try:
                return fn(*args, **kw)
            finally:
                b.record()
                self.depth -= 1
                self.records.append((label, flops, a, b))

        self.saved.append((module, name, fn))
        setattr(module, name, timed)

    def install(self):
        from . import ops
        from .ops import attention
        for name in dir(ops):
            f = getattr(ops, name)
            if callable(f) and getattr(f, "__module__", "") == ops.__name__ and not name.startswith("_") and \
                    name not in ("lib", "check", "stream_ptr", "ptr", "device_error", "clear_device_error",
                                 "KernelError"):
                self.wrap(ops, name)
        for name in ("attention_fwd", "attention_bwd"):
            self.wrap(attention, name)

    def uninstall(self):
        for module, name, fn in reversed(self.saved):
            setattr(module, name, fn)
        self.saved = []

    def summary(self):
        torch.cuda.synchronize()
        agg = collections.OrderedDict()
        for label, flops, a, b in self.records:
            ms = a.elapsed_time(b)
            e = agg.setdefault(label, [0, 0.0, 0.0])
            e[0] += 1
            e[1] += ms
            e[2] += flops
        return agg


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="tiny")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args()
    sys.path.insert(0, ROOT)
    from .config import bench_config
    from .models.engine import TrainEngine
    from .bench_kernels import peaks
    run = bench_config(args.config)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    eng = TrainEngine(run.model, run.micro_batch, run.seq_len, optim=run.optim, device=dev, seed=run.seed,
                      init_std=run.init_std, act_ckpt=run.activation_checkpointing)
    g = torch.Generator().manual_seed(7)
    eng.set_tokens(torch.randint(0, run.model.vocab_size, (run.micro_batch, run.seq_len), generator=g,
                                 dtype=torch.int32).to(dev))
    for _ in range(args.warmup):
        eng.step_kernels()
    torch.cuda.synchronize()
    # whole step, eager and graph-replayed
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        eng.step_kernels()
    e.record()
    torch.cuda.synchronize()
    eager_ms = s.elapsed_time(e) / args.steps
    eng.capture()
    for _ in range(2):
        eng.step()
    torch.cuda.synchronize()
    s.record()
    for _ in range(args.steps):
        eng.step()
    e.record()
    torch.cuda.synchronize()
    graph_ms = s.elapsed_time(e) / args.steps
    eng.release_graph()
    # per call
    t = CallTimer()
    t.install()
    try:
        for _ in range(args.steps):
            eng.step_kernels()
        agg = t.summary()
    finally:
        t.uninstall()
    pk = peaks()
    rows = []
    total = 0.0
    for label, (calls, ms, flops) in agg.items():
        ms /= args.steps
        calls //= args.steps
        flops /= args.steps
        total += ms
        row = {"call": label, "calls_per_step": calls, "ms_per_step": round(ms, 4)}
        if flops:
            tf = flops / (ms * 1e-3) / 1e12
            row["tflops"] = round(tf, 1)
            row[f"frac_of_{pk['src']}_sustained_bf16"] = round(tf / pk["bf16_tflops_sustained"], 3)
        rows.append(row)
    rows.sort(key=lambda r: -r["ms_per_step"])
    for r in rows:
        r["share_of_step"] = round(r["ms_per_step"] / graph_ms, 4)
    out = {"config": f"{run.name} B{run.micro_batch} S{run.seq_len}", "graph_step_ms": round(graph_ms, 3),
           "eager_step_ms": round(eager_ms, 3), "sum_of_calls_ms": round(total, 3),
           "gemm_ms": round(sum(r["ms_per_step"] for r in rows if "tflops" in r and not r["call"].startswith("attention")), 3),
           "attention_ms": round(sum(r["ms_per_step"] for r in rows if r["call"].startswith("attention")), 3),
           "calls": rows}
    if args.json:
        print(json.dumps(out))
        return
    print(f"{out['config']}: graph step {graph_ms:.3f} ms, eager {eager_ms:.3f} ms, sum of timed calls "
          f"{total:.3f} ms (GEMMs {out['gemm_ms']:.3f}, attention {out['attention_ms']:.3f})")
    print(f"{'call':58s} {'n':>3s} {'ms/step':>9s} {'share':>6s} {'TFLOP/s':>8s}")
    for r in rows:
        print(f"{r['call'][:58]:58s} {r['calls_per_step']:3d} {r['ms_per_step']:9.3f} {r['share_of_step']:6.3f} "
              f"{r.get('tflops', ''):>8}")


if __name__ == "__main__":
    main()
