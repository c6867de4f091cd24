"""Roofline figures for the benchmark JSON lines, against the peaks measured on this pool's B200s
(``MEASURED_PEAKS.json``: STREAM-style copy bandwidth and cuBLAS bf16 throughput, burst and sustained;
an 8-rank peer copy of 770 GB/s per direction for NVLink).

* training step: model FLOPs per token = 6 N (forward + backward of every weight, the tied LM head
  included once) + 6 L S H (causal attention scores and values over S positions, forward + backward)
  + 2 N' with activation checkpointing (the recomputed block forwards, N' = non-embedding weights);
  achieved TFLOP/s per GPU against the sustained bf16 peak (a step is seconds of back-to-back GEMMs
  under the power cap);
* merge: the slowest GPU's bytes over NVLink at the measured peer-copy rate and its HBM bytes at the
  measured copy bandwidth; the roofline time is the larger of the two, reported as a fraction of the
  measured merge time.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Optional

NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool (nominal 900)
_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


def peaks(path: Optional[str] = None) -> Dict[str, float]:
    """Measured peaks (``src`` = "measured"), or the pool's earlier figures (``src`` = "fallback")."""
    path = path or os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "src": "measured"}
    except (OSError, KeyError, ValueError):
        return dict(_FALLBACK)


def train_flops_per_token(cfg, seq_len: int, act_ckpt: bool = False) -> float:
    n = cfg.param_count()
    emb = cfg.vocab_size * cfg.hidden_dim
    f = 6.0 * n + 6.0 * cfg.num_layers * seq_len * cfg.hidden_dim
    if act_ckpt:
        f += 2.0 * (n - emb)
    return f


def step_roofline(cfg, seq_len: int, tokens_per_s: float, n_gpus: int, act_ckpt: bool = False,
                  pk: Optional[Dict[str, float]] = None) -> Dict[str, float]:
    pk = pk or peaks()
    tf = tokens_per_s * train_flops_per_token(cfg, seq_len, act_ckpt) / max(n_gpus, 1) / 1e12
    return {"model_tflops_per_gpu": round(tf, 1),
            f"frac_of_{pk['src']}_sustained_bf16": round(tf / pk["bf16_tflops_sustained"], 3),
            f"frac_of_{pk['src']}_burst_bf16": round(tf / pk["bf16_tflops"], 3)}


def distributed_merge_roofline(n_params: int, payload_bytes: float, n_nodes: int, merge_ms: float,
                               multicast: bool = True, pk: Optional[Dict[str, float]] = None) -> Dict[str, float]:
    """Per GPU of a W-node distributed merge, W members of ``payload_bytes`` each (s = 4 n / W, one slice):
    NVLink in  = (W-1) P/W (its slice of every remote payload) + (W-1) s (the other nodes' slices);
    NVLink out = (W-1) P/W (peers read its payload) + s (multicast; (W-1) s with per-peer stores);
    HBM        = 2 s (its slice read and written) + P (its payload, read by itself and the peers)
                 + (W-1) s (the other slices landing in its staging buffer)."""
    pk = pk or peaks()
    W = max(n_nodes, 1)
    s = n_params * 4.0 / W
    P = float(payload_bytes)
    nvlink_in = (W - 1) * (P / W + s)
    nvlink_out = (W - 1) * P / W + s * (1 if multicast else W - 1) if W > 1 else 0.0
    nvlink = max(nvlink_in, nvlink_out)
    hbm = 2 * s + P + (W - 1) * s
    t_link = nvlink / (NVLINK_GBS * 1e9) * 1e3
    t_hbm = hbm / (pk["hbm_gbs"] * 1e9) * 1e3
    t = max(t_link, t_hbm)
    return {"nvlink_bytes_per_gpu": int(nvlink), "hbm_bytes_per_gpu": int(hbm), "roofline_ms": round(t, 3),
            "bound": "nvlink" if t_link >= t_hbm else "hbm",
            f"frac_of_{pk['src']}": round(t / merge_ms, 3) if merge_ms > 0 else None}
