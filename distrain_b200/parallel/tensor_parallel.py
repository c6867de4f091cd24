"""Tensor parallelism for one model replica over a small group of GPUs (TP=2 for the large preset).

Megatron-style split of every transformer block (no sequence parallelism):

* column-parallel: the fused QKV weight (and bias) by attention head, and the fused gate|up weight by
  FFN row - each rank holds ``num_heads / tp`` query heads, ``num_kv_heads / tp`` kv heads and
  ``ffn_hidden_dim / tp`` FFN rows; attention and SwiGLU run on local heads / rows with no traffic;
* row-parallel: o_proj and down_proj by input column - each rank produces a partial sum of the full
  ``[tokens, hidden]`` output, which is all-reduced over the group;
* replicated: embedding (tied LM head), every RMSNorm weight, the output scale. The residual stream is
  replicated, so these parameters see identical gradients on every rank and need no gradient traffic.

Per block and step that is two all-reduces in the forward (after o_proj and down_proj) and two in the
backward (after the QKV and gate|up data-gradient GEMMs), plus one tiny all-reduce of the per-tensor
gradient norms for clipping. ``TensorParallel`` issues them on the current stream through NCCL (the
correctness path, also capturable in a CUDA graph) or, in ``fused`` mode, the GEMM epilogues store
their partial tiles straight into the peer's receive buffer over NVLink and the consuming norm kernel
adds both partials (``dt_gemm_bf16_peer`` / ``dt_add_rmsnorm_fwd_tp`` / ``dt_rmsnorm_bwd_tp``).

There is no tensor parallelism in the reference (node/cli/src/trainer.rs and the Burn model in
core/model/src/model.rs train one replica per device); the split follows the parameter names of
``core/model/src/model.rs:401-467`` so checkpoints gather back into the reference's state dict.
"""
from __future__ import annotations

import zlib
from typing import Dict, List

import torch
import torch.distributed as dist

from ..config import ModelConfig

_COL = (".q_proj.", ".k_proj.", ".v_proj.", ".gate_proj.", ".up_proj.")   # split along dim 0 (rows)
_ROW = (".o_proj.", ".down_proj.")                                       # split along dim 1 (columns)


def split_dim(name: str):
    """0 (output rows), 1 (input columns) or None (replicated) for a parameter name."""
    if any(k in name for k in _COL):
        return 0
    if any(k in name for k in _ROW) and name.endswith(".weight"):
        return 1
    return None


def shard_state_dict(full: Dict[str, torch.Tensor], cfg: ModelConfig, rank: int, size: int) -> Dict[str, torch.Tensor]:
    """The rank's slice of a full (reference-named) state dict."""
    out = {}
    for k, v in full.items():
        dim = split_dim(k)
        if dim is None:
            out[k] = v
        else:
            n = v.shape[dim] // size
            out[k] = v.narrow(dim, rank * n, n).contiguous()
    return out


def gather_state_dict(shards: List[Dict[str, torch.Tensor]]) -> Dict[str, torch.Tensor]:
    """Inverse of ``shard_state_dict`` (rank order)."""
    out = {}
    for k, v in shards[0].items():
        dim = split_dim(k)
        out[k] = v if dim is None else torch.cat([s[k] for s in shards], dim=dim)
    return out


def norm_weights(layout, device) -> torch.Tensor:
    """Per-segment factor applied to the local squared gradient norms before the group sum: 1 for split
    tensors (the halves add up to the full norm), 1/size for replicated ones (identical on every rank)."""
    w = [1.0 if split_dim(e.name) is not None else 1.0 / layout.tp_size for e in layout.entries]
    return torch.tensor(w, dtype=torch.float32, device=device)


def init_flat_tp(layout, std: float = 0.02, seed: int = 0, device="cuda") -> torch.Tensor:
    """Seeded N(0, std) init of this rank's shard, generated on the device. Replicated tensors use a
    generator keyed by (seed, name) only, so they are identical on every rank; split tensors add the rank."""
    flat = torch.zeros(layout.total, dtype=torch.float32, device=device)
    g = torch.Generator(device=device)
    for e in layout.entries:
        v = flat[e.offset:e.offset + e.numel]
        if e.name.endswith("norm.weight") or e.name.endswith("output_scale"):
            v.fill_(1.0)
        elif e.name.endswith(".bias"):
            v.zero_()
        else:
            key = zlib.crc32(e.name.encode()) ^ (seed * 0x9E3779B1)
            if split_dim(e.name) is not None:
                key ^= (layout.tp_rank + 1) * 0x85EBCA77
            g.manual_seed(key & 0x7FFFFFFFFFFFFFFF)
            v.copy_(torch.randn(e.numel, generator=g, device=device) * std)
    return flat


class TensorParallel:
    """One tensor-parallel group as seen by one rank; the engine calls these hooks on its stream.

    ``mode="nccl"``: partial sums are all-reduced with NCCL between the producing GEMM and its consumer.
    ``mode="fused"`` (TP=2): the producing GEMM stores every output box into the peer's receive buffer
    over NVLink as it is computed and signals an arrival counter; the consuming norm kernel adds the
    local and the received partial after a bounded wait. The receive buffers (three [rows, hidden] bf16
    slots) and counters live in one symmetric allocation; ``slots_per_step`` ops of one training step
    use slots 0/1 alternately and, when their count is odd, slot 2 for the last one, so consecutive ops
    (across CUDA-graph replays too) never share a slot: a rank can run at most one op ahead of its peer,
    because every consumer waits for the peer's matching producer."""

    COUNTERS = 4096  # bytes: arrivals @0, consumed @128, done_ctas @256, done_blocks @384

    def __init__(self, group, rank: int, size: int, mode: str = "nccl", rows: int = 0, hidden: int = 0,
                 device=None):
        self.group, self.rank, self.size = group, rank, size
        self.mode = mode if size > 1 else "nccl"
        self.fused = self.mode == "fused"
        self.slots_per_step = 0
        self._j = 0
        if self.fused:
            assert size == 2, "the fused exchange is written for TP=2"
            import torch.distributed._symmetric_memory as symm_mem
            self.rows, self.hidden = rows, hidden
            self.slot_bytes = (rows * hidden * 2 + 4095) // 4096 * 4096
            nbytes = self.COUNTERS + 3 * self.slot_bytes
            self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
            self.buf.zero_()
            self.hdl = symm_mem.rendezvous(self.buf, group.group_name)
            torch.cuda.synchronize()
            dist.barrier(group=group)
            base = self.buf.data_ptr()
            self.peer_base = int(self.hdl.buffer_ptrs[1 - rank])
            self.arrivals, self.consumed = base, base + 128
            self.done_ctas, self.done_blocks = base + 256, base + 384
            self.peer_arrivals = self.peer_base

    # ── fused-mode slot bookkeeping (host side, fixed per step, so graph replays repeat it) ──
    def begin_step(self, slots_per_step: int):
        self.slots_per_step = slots_per_step
        self._j = 0

    def next_slot(self) -> int:
        j, n = self._j, self.slots_per_step
        self._j += 1
        return 2 if (n % 2 == 1 and j == n - 1) else j % 2

    def recv(self, slot: int) -> torch.Tensor:
        off = self.COUNTERS + slot * self.slot_bytes
        return self.buf[off:off + self.rows * self.hidden * 2].view(torch.bfloat16).view(self.rows, self.hidden)

    def peer_recv_ptr(self, slot: int) -> int:
        return self.peer_base + self.COUNTERS + slot * self.slot_bytes

    # ── NCCL path ──
    def allreduce_(self, t: torch.Tensor, slot: str = "", layer: int = 0):
        if self.size > 1:
            dist.all_reduce(t, group=self.group)

    def sum_norms_(self, norms: torch.Tensor, weights: torch.Tensor):
        if self.size > 1:
            norms.mul_(weights)
            dist.all_reduce(norms, group=self.group)
