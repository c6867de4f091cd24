"""Kernel microbenchmarks: CUDA-event timing of the hot sm_100a kernels on the tiny/small preset shapes.

    python -m distrain_b200.bench_kernels [--only gemm|attn|norm|fused|compress|merge|all] [--case SUBSTR] [--iters N]
                                          [--warmup W] [--json]

``--case`` keeps only the cases whose name contains SUBSTR (e.g. ``gate_up_fwd``, ``attn_fwd_d64``,
``rmsnorm_bwd``, ``compress_10``, ``merge_10``); with ``--iters 1 --warmup 1`` a case launches its kernel twice, which
is what a single-launch profiler capture wants.

Each case runs warm-up launches, then ``iters`` launches between two events on the launching stream
(synchronised on both sides); inputs are resized so every case reads more than the 126 MB L2, or the
case is marked ``l2_resident``. Reported: time per launch, achieved TFLOP/s or GB/s, and the fraction of
the measured peaks in MEASURED_PEAKS.json ("of measured") or the recorded fallback figures.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


_CASE = None
_WARMUP = 3


def want(name: str) -> bool:
    return _CASE is None or _CASE in name


def time_it(fn, iters=20, warmup=None):
    warmup = _WARMUP if warmup is None else min(warmup, _WARMUP)
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def gemm_cases(iters):
    from distrain_b200 import ops
    pk = peaks()
    out = []
    M = 32736
    shapes = [  # name, M, N, K, a_mn, b_mn, epi
        ("qkv_fwd", M, 1280, 768, 0, 0, 0), ("o_fwd", M, 768, 768, 0, 0, 0), ("gate_up_fwd", M, 4096, 768, 0, 0, 0),
        ("down_fwd", M, 768, 2048, 0, 0, 0), ("lm_head_fwd_chunk", 8192, 32768, 768, 0, 0, 0),
        ("gate_up_dgrad", M, 768, 4096, 0, 1, 0), ("down_dgrad", M, 2048, 768, 0, 1, 0),
        ("gate_up_wgrad", 4096, 768, M, 1, 1, 2), ("down_wgrad", 768, 2048, M, 1, 1, 2),
        ("qkv_wgrad", 1280, 768, M, 1, 1, 2), ("lm_head_wgrad_chunk", 32768, 768, 8192, 1, 1, 2),
        ("lm_head_dgrad_chunk", 8192, 768, 32768, 0, 1, 0), ("square_8192", 8192, 8192, 8192, 0, 0, 0),
    ]
    for name, m, n, k, a_mn, b_mn, epi in shapes:
        if not want(name):
            continue
        A = torch.randn(k if a_mn else m, m if a_mn else k, device="cuda").bfloat16()
        B = torch.randn(k if b_mn else n, n if b_mn else k, device="cuda").bfloat16()
        C = torch.zeros(m, n, device="cuda", dtype=torch.bfloat16 if epi == 0 else torch.float32)
        fn = lambda: ops.gemm(A, B, C, M=m, N=n, K=k, a_mn=bool(a_mn), b_mn=bool(b_mn), epi=epi)
        ms = time_it(fn, iters)
        tf = 2.0 * m * n * k / (ms * 1e-3) / 1e12
        out.append({"kernel": "gemm_tc", "case": name, "M": m, "N": n, "K": k, "ms": round(ms, 4),
                    "tflops": round(tf, 1), f"frac_of_{pk['src']}_bf16": round(tf / pk["bf16_tflops"], 3)})
        del A, B, C
    return out


def attn_cases(iters):
    from distrain_b200.ops import attention as A
    pk = peaks()
    out = []
    for (B, T, nh, nkv, d) in [(32, 1023, 12, 4, 64), (8, 2047, 16, 4, 128)]:
        do_f, do_b = want(f"attn_fwd_d{d}"), want(f"attn_bwd_d{d}")
        if not (do_f or do_b or want(f"attn_bwd_ds_d{d}")):
            continue
        W = (nh + 2 * nkv) * d
        qkv = torch.randn(B * T, W, device="cuda").bfloat16()
        o = torch.empty(B * T, nh * d, device="cuda", dtype=torch.bfloat16)
        lse = torch.empty(B, nh, A.lse_stride(T), device="cuda")
        do = torch.randn_like(o)
        dqkv = torch.empty_like(qkv)
        dqa = torch.empty(B * T, nh * d, device="cuda")
        de = torch.empty(B, nh, A.lse_stride(T), device="cuda")
        fl = 4.0 * B * nh * T * T * d / 2  # causal
        A.attention_fwd(qkv, o, lse, B=B, T=T, nh=nh, nkv=nkv, d=d)  # valid LSE for the backward
        ms_f = time_it(lambda: A.attention_fwd(qkv, o, lse, B=B, T=T, nh=nh, nkv=nkv, d=d), iters) if do_f else None
        ms_b = time_it(lambda: A.attention_bwd(qkv, o, do, lse, dqkv, dqa, de, B=B, T=T, nh=nh, nkv=nkv, d=d),
                       iters) if do_b else None
        ms_bd = None
        if want(f"attn_bwd_ds_d{d}"):  # dS^T stored once, dQ from it (the engine's path)
            dsb = torch.empty(A.ds_bytes(B, T, nh), dtype=torch.uint8, device="cuda")
            ms_bd = time_it(lambda: A.attention_bwd(qkv, o, do, lse, dqkv, dqa, de, B=B, T=T, nh=nh, nkv=nkv, d=d,
                                                    ds_buf=dsb), iters)
            del dsb
        for nm, ms, f in (("fwd", ms_f, fl), ("bwd", ms_b, 2.5 * fl), ("bwd_ds", ms_bd, 2.5 * fl)):
            if ms is None:
                continue
            tf = f / (ms * 1e-3) / 1e12
            out.append({"kernel": f"attn_{nm}", "case": f"B{B} T{T} h{nh}/{nkv} d{d}", "ms": round(ms, 4),
                        "tflops": round(tf, 1), f"frac_of_{pk['src']}_bf16": round(tf / pk["bf16_tflops"], 3)})
    return out


def norm_cases(iters):
    from distrain_b200 import ops
    pk = peaks()
    M, H = 32736, 768
    x = torch.randn(M, H, device="cuda")
    br = torch.randn(M, H, device="cuda").bfloat16()
    w = torch.ones(H, device="cuda")
    r = torch.empty(M, H, device="cuda")
    y = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    rs = torch.empty(M, device="cuda")
    out = []
    if want("add_rmsnorm_fwd") or want("rmsnorm_bwd"):
        ms = time_it(lambda: ops.add_rmsnorm_fwd(x=x, br=br, w=w, out_resid=r, y=y, rstd=rs, eps=1e-5, M=M, H=H),
                     iters)
        byt = M * H * (4 + 2 + 4 + 2)
        if want("add_rmsnorm_fwd"):
            out.append({"kernel": "add_rmsnorm_fwd", "case": f"{M}x{H}", "ms": round(ms, 4),
                        "gbs": round(byt / ms / 1e6, 1),
                        f"frac_of_{pk['src']}_hbm": round(byt / ms / 1e6 / pk["hbm_gbs"], 3)})
    if not want("rmsnorm_bwd"):
        return out
    dres = torch.zeros(M, H, device="cuda")
    d16 = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    dw = torch.zeros(H, device="cuda")
    ms = time_it(lambda: ops.rmsnorm_bwd(dy=y, x=r, rstd=rs, w=w, dresid_in=dres, dresid_out=dres, dresid16=d16, dw=dw,
                                         M=M, H=H), iters)
    byt = M * H * (2 + 4 + 4 + 4 + 2)
    out.append({"kernel": "rmsnorm_bwd", "case": f"{M}x{H}", "ms": round(ms, 4), "gbs": round(byt / ms / 1e6, 1),
                f"frac_of_{pk['src']}_hbm": round(byt / ms / 1e6 / pk["hbm_gbs"], 3)})
    return out


def fused_cases(iters):
    """Fused epilogues against the separate kernels they replace, on the tiny preset's layer shapes:
    gate|up GEMM + SwiGLU, down data-gradient + SwiGLU backward, QKV GEMM + bias + RoPE; and AdamW."""
    from distrain_b200 import ops
    from distrain_b200.config import preset
    from distrain_b200.models.oracle import rope_tables
    pk = peaks()
    out = []
    M, H, F, T = 32736, 768, 2048, 1023
    x = torch.randn(M, H, device="cuda").bfloat16()
    wgu = (torch.randn(2 * F, H, device="cuda") * 0.03).bfloat16()
    gu = torch.empty(M, 2 * F, device="cuda", dtype=torch.bfloat16)
    h = torch.empty(M, F, device="cuda", dtype=torch.bfloat16)

    def rec(name, ms, flops=None, byt=None):
        r = {"kernel": name, "case": "tiny layer", "ms": round(ms, 4)}
        if flops:
            r["tflops"] = round(flops / ms / 1e9, 1)
        if byt:
            r["gbs"] = round(byt / ms / 1e6, 1)
            r[f"frac_of_{pk['src']}_hbm"] = round(byt / ms / 1e6 / pk["hbm_gbs"], 3)
        out.append(r)
    fl = 2.0 * M * 2 * F * H
    if want("swiglu_fwd"):
        rec("gemm_swiglu_fwd (fused)", time_it(lambda: ops.gemm_swiglu_fwd(x, wgu, gu, h), iters), fl)
        rec("linear_fwd + swiglu_fwd (separate)",
            time_it(lambda: (ops.linear_fwd(x, wgu, gu), ops.swiglu_fwd(gu, h, M=M, F=F)), iters), fl)
    if want("swiglu_bwd"):
        dy = torch.randn(M, H, device="cuda").bfloat16()
        wd = (torch.randn(H, F, device="cuda") * 0.03).bfloat16()
        dgu = torch.empty_like(gu)
        dh = torch.empty(M, F, device="cuda", dtype=torch.bfloat16)
        fb = 2.0 * M * F * H
        rec("gemm_swiglu_bwd (fused)", time_it(lambda: ops.gemm_swiglu_bwd(dy, wd, gu, dgu), iters), fb)
        rec("linear_dgrad + swiglu_bwd (separate)",
            time_it(lambda: (ops.linear_dgrad(dy, wd, dh), ops.swiglu_bwd(dh, gu, dgu, M=M, F=F)), iters), fb)
    if want("qkv_rope"):
        cfg = preset("tiny")
        nh, nkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim()
        W = (nh + 2 * nkv) * d
        wq = (torch.randn(W, H, device="cuda") * 0.03).bfloat16()
        b = torch.zeros(W, device="cuda")
        cos, sin = rope_tables(cfg, T)
        cos, sin = cos.cuda().contiguous(), sin.cuda().contiguous()
        q = torch.empty(M, W, device="cuda", dtype=torch.bfloat16)
        fq = 2.0 * M * W * H
        rec("gemm_qkv_rope (fused)", time_it(lambda: ops.gemm_qkv_rope(x, wq, b, cos, sin, q, T=T, d=d,
                                                                     rot_cols=(nh + nkv) * d), iters), fq)
        rec("linear_fwd + rope_fwd (separate)",
            time_it(lambda: (ops.linear_fwd(x, wq, q), ops.rope_fwd(q, b, cos, sin, M=M, T=T, nh=nh, nkv=nkv, d=d)),
                    iters), fq)
    if want("rope_bwd"):
        cfg = preset("tiny")
        nh, nkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim()
        W = (nh + 2 * nkv) * d
        cos, sin = rope_tables(cfg, T)
        cos, sin = cos.cuda().contiguous(), sin.cuda().contiguous()
        dq = (torch.randn(M, W, device="cuda") * 0.1).bfloat16()
        db = torch.zeros(W, device="cuda")
        part = torch.empty(ops.rope_bwd_scratch(M, nh, nkv, d), device="cuda")
        ms = time_it(lambda: ops.rope_bwd(dq, db, cos, sin, M=M, T=T, nh=nh, nkv=nkv, d=d, part=part), iters)
        gbs = 2 * M * W * 2 / ms / 1e6
        out.append({"kernel": "rope_bwd", "case": f"M{M} W{W} (inverse rotation + bias gradient)", "ms": round(ms, 4),
                    "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / pk["hbm_gbs"], 3)})
    if want("adamw"):
        from distrain_b200.models.params import ParamLayout
        L = ParamLayout(preset("tiny"))
        n = L.total
        p32 = torch.randn(n, device="cuda") * 0.02
        g = torch.randn(n, device="cuda") * 1e-3
        m = torch.zeros(n, device="cuda")
        v = torch.zeros(n, device="cuda")
        p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
        cseg, cstart, cend, nseg = L.chunk_tables(torch.device("cuda"))
        norms = torch.zeros(nseg, device="cuda")
        hp = torch.tensor([3e-4, 0.9, 0.999, 1e-5, 0.1, 0, 0, 1.0, 0, 0, 0, 1.0, 0, 0, 0, 0], device="cuda")
        rec("adamw_step (clears gradients)", time_it(lambda: ops.adamw_step(p32, g, m, v, p16, cseg, cstart, cend, norms,
                                                                            hp), iters), None, 34 * n)
        hp[11] = 0.0
        rec("adamw_step (keeps gradients)", time_it(lambda: ops.adamw_step(p32, g, m, v, p16, cseg, cstart, cend, norms,
                                                                           hp), iters), None, 30 * n)
    return out


def compress_cases(iters):
    from distrain_b200.config import preset, CompressionConfig
    from distrain_b200.models.params import ParamLayout
    from distrain_b200.parallel.compression import DeviceCompressor
    pk = peaks()
    out = []
    for name, k in (("tiny", 0.01), ("tiny", 0.10), ("tiny", 0.99)):
        if not want(f"compress_{round(k * 100)}"):
            continue
        L = ParamLayout(preset(name))
        comp = DeviceCompressor(L, torch.device("cuda"), CompressionConfig(top_k_fraction=k, int8_block=256))
        master = torch.randn(L.total, device="cuda") * 1e-2
        comp.snap.copy_(master + torch.randn_like(master) * 1e-4)
        ms = time_it(lambda: (comp.begin(master), comp.finish()), iters, warmup=2)
        out.append({"kernel": "compress_pipeline", "case": f"{name} {L.num_params()/1e6:.0f}M top-k {k:.0%}",
                    "ms": round(ms, 3), "gbs_effective": round(L.total * 4 * 6 / ms / 1e6, 1)})
    return out


def merge_cases(iters):
    """Coordinator merge of 8 compressed deltas of the tiny model held in this GPU's memory (the same
    kernels read peer memory in the multi-GPU run): prepass (validation norms) + weighted dequant
    scatter-add into the checkpoint + fp32 broadcast to one destination's staging buffer. Reported per
    merge, including the host round trip of the prepass."""
    from distrain_b200.config import preset, CompressionConfig
    from distrain_b200.models.params import ParamLayout
    from distrain_b200.parallel.compression import DeviceCompressor, DevicePayload
    from distrain_b200.parallel.merge import DeviceMerger, Contribution
    out = []
    L = ParamLayout(preset("tiny"))
    dev = torch.device("cuda")
    for k in (0.01, 0.10, 0.99):
        if not want(f"merge_{round(k * 100)}"):
            continue
        comp = DeviceCompressor(L, dev, CompressionConfig(top_k_fraction=k, int8_block=256))
        master = torch.randn(L.total, device=dev) * 1e-2
        pays, contribs = [], []
        for i in range(8):
            comp.reset(master)
            comp.begin(master - torch.randn_like(master) * 1e-4)
            p = DevicePayload.allocate(comp.capacity, 256, dev)
            comp.finish(payload=p)
            torch.cuda.synchronize()
            cnt = int(comp.stats_host[comp.nseg * 6].item())
            pays.append(p)
            contribs.append(Contribution(idx_ptr=p.idx.data_ptr(), q_ptr=p.q.data_ptr(), val_ptr=p.val.data_ptr(),
                                         win_ptr=p.win.data_ptr(),
                                         scales_ptr=p.scales.data_ptr(), count=cnt, block=256, dense=False,
                                         weight=1000.0 * (i + 1), wire_bytes=cnt * 5 + (cnt + 255) // 256 * 4))
        m = DeviceMerger(L.total, dev, master)
        s32 = torch.empty(L.total, device=dev)  # one destination node's staging buffer

        def run():
            m.merge(contribs, 1.0, stage32=[s32.data_ptr()])
            m.stream.synchronize()
        ms = time_it(run, iters, warmup=2)
        wire = sum(c.wire_bytes for c in contribs)
        out.append({"kernel": "merge_pipeline", "case": f"8 x tiny {L.num_params() / 1e6:.0f}M top-k {k:.0%}",
                    "ms": round(ms, 3), "payload_mb": round(wire / 1e6, 1)})
        del comp, m, pays, s32
    return out


def dm_cases(iters):
    """The distributed merge's kernels on one GPU (one node owning the whole range, so no broadcast): per
    merge, the range search over 8 payloads of the tiny model and the weighted dequant scatter-add into the
    checkpoint (global atomics), or the fused tile pass that sums the payloads per 8192-element tile in
    shared memory and updates the checkpoint once. Plans come from the reported statistics (no device pass over the payloads)."""
    from distrain_b200.config import preset, CompressionConfig
    from distrain_b200.models.params import ParamLayout
    from distrain_b200.parallel.compression import DeviceCompressor, DevicePayload
    from distrain_b200.parallel.merge import DeviceMerger, DistributedMerger, Contribution
    out = []
    L = ParamLayout(preset("tiny"))
    dev = torch.device("cuda")
    for k in (0.01, 0.10, 0.99):
        if not want(f"dm_{round(k * 100)}"):
            continue
        comp = DeviceCompressor(L, dev, CompressionConfig(top_k_fraction=k, int8_block=256))
        master = torch.randn(L.total, device=dev) * 1e-2
        pays, contribs, stats = [], [], []
        for i in range(8):
            comp.reset(master)
            comp.begin(master - torch.randn_like(master) * 1e-4)
            p = DevicePayload.allocate(comp.capacity, 256, dev)
            comp.finish(payload=p)
            torch.cuda.synchronize()
            st = comp.read_stats()
            cnt = st["num_params_kept"]
            pays.append(p)
            stats.append(st["wire"])
            contribs.append(Contribution(idx_ptr=p.idx.data_ptr(), q_ptr=p.q.data_ptr(), val_ptr=p.val.data_ptr(),
                                         win_ptr=p.win.data_ptr(), scales_ptr=p.scales.data_ptr(), count=cnt,
                                         block=256, dense=False, weight=1000.0 * (i + 1),
                                         wire_bytes=p.wire_bytes(cnt)))
        theta = master.clone()
        ctl = torch.zeros(DistributedMerger.CTL_BYTES, dtype=torch.uint8, device=dev)
        dm = DistributedMerger(0, 1, L.total, dev, theta, [theta.data_ptr()], 0, ctl, [ctl.data_ptr()])
        coefs, _ = DeviceMerger.plan(contribs, stats)
        torch.cuda.synchronize()

        def run():
            dm.apply(contribs, coefs, 1.0)
            dm.stream.synchronize()
        wire = sum(c.wire_bytes for c in contribs)
        for fused in (False, True):  # scatter-add into the checkpoint, or the tile-sum pass (dt_dm_fused)
            dm.fused = fused
            ms = time_it(run, iters, warmup=2)
            out.append({"kernel": "dm_fused_tiles" if fused else "dm_range_apply",
                        "case": f"8 x tiny {L.num_params() / 1e6:.0f}M top-k {k:.0%}",
                        "ms": round(ms, 3), "payload_mb": round(wire / 1e6, 1),
                        "payload_gbs": round(wire / ms / 1e6, 1)})
        del comp, dm, pays, theta
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="all")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--case", default=None)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    global _CASE, _WARMUP
    _CASE, _WARMUP = a.case, a.warmup
    sys.path.insert(0, ROOT)
    res = []
    sel = a.only.split(",")
    if "all" in sel or "gemm" in sel:
        res += gemm_cases(a.iters)
    if "all" in sel or "attn" in sel:
        res += attn_cases(a.iters)
    if "all" in sel or "norm" in sel:
        res += norm_cases(a.iters)
    if "all" in sel or "fused" in sel:
        res += fused_cases(a.iters)
    if "all" in sel or "compress" in sel:
        res += compress_cases(a.iters)
    if "all" in sel or "merge" in sel:
        res += merge_cases(a.iters)
    if "all" in sel or "dm" in sel:
        res += dm_cases(a.iters)
    from distrain_b200 import ops
    code, site = ops.device_error()
    for r in res:
        print(json.dumps(r) if a.json else "  ".join(f"{k}={v}" for k, v in r.items()))
    if code:
        print(f"DEVICE ERROR {code} at {site}")
        sys.exit(1)


if __name__ == "__main__":
    main()
