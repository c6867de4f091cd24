"""Device-memory estimate of one in-box node rank, from the sizes of the buffers the engine and the protocol
allocate (the in-box counterpart of the reference's VRAM batch estimate, node/cli/src/trainer.rs:163-230):

* engine: fp32 master, gradients and AdamW moments, bf16 compute copy (18 B per local parameter), the
  per-layer residual inputs (all layers with activation checkpointing, plus the per-block buffers of
  one block; every block's buffers without it) and the LM-head chunk;
* protocol: round-start snapshot and error feedback (8 B per parameter), one fp32 staging slot (4 B),
  the payload slots (9 B per kept entry at the largest top-k, or 4 B per parameter for raw
  bandwidth-adaptive pushes).

The large preset (TP=2 x 4 nodes, activation checkpointing, one payload slot) is estimated at 184.5 GB
per rank and measured at 188.3 GB (CUDA context, NCCL and allocator slack make up the rest).
"""
from __future__ import annotations

from typing import Dict


def estimate_rank_bytes(run, n_nodes: int = 1, protocol: bool = True) -> Dict[str, float]:
    from .models.params import ParamLayout
    from .parallel.compression import DeviceCompressor, DevicePayload
    m = run.model
    tp = max(int(run.tp), 1)
    L = ParamLayout(m, 0, tp) if tp > 1 else ParamLayout(m)
    n = L.total
    B, S = run.micro_batch, run.seq_len
    M = B * (S - 1)
    H = m.hidden_dim
    F = m.ffn_hidden_dim // tp
    nh, nkv = m.num_heads // tp, max(m.num_kv_heads // tp, 1)
    d = H // m.num_heads
    W = (nh + 2 * nkv) * d
    per_block = (M * H * 4 + 2 * M * 4 + 2 * M * H * 2 + M * W * 2 + M * nh * d * 2 + B * nh * S * 4 +
                 M * 2 * F * 2 + M * F * 2)
    blocks = 1 if run.activation_checkpointing else m.num_layers
    act = (m.num_layers * M * H * 4 + blocks * per_block + M * H * (4 + 4 + 2 + 2 + 2 + 2) + M * 4 * 2 +
           min(M, 32768) * m.vocab_size * 2 + M * F * 2 + M * 2 * F * 2 + M * nh * d * (2 + 4) + M * W * 2)
    out = {"params_local": n, "engine": 18.0 * n, "activations": float(act), "protocol": 0.0}
    if protocol and n_nodes >= 1:
        cfg = run.compression
        kmax = max(cfg.top_k_fraction, 0.80 if run.bandwidth_adaptive else 0.0)
        blk = cfg.int8_block if cfg.quantize_int8 else 0
        slot = DevicePayload.nbytes(DeviceCompressor.capacity_for(L, kmax), blk)
        if run.bandwidth_adaptive:
            slot = max(slot, 4 * n)
        out["protocol"] = 12.0 * n + max(1, int(run.payload_slots)) * float(slot)
    out["total"] = out["engine"] + out["activations"] + out["protocol"]
    return out


def check_fits(run, device_bytes: float, n_nodes: int = 1, protocol: bool = True, margin: float = 0.97):
    """(fits, estimate): the estimate against `margin` of the device's memory."""
    est = estimate_rank_bytes(run, n_nodes, protocol)
    return est["total"] <= margin * device_bytes, est
