"""Flat parameter layout.

All parameters of a model live in ONE contiguous fp32 buffer (the master copy), with named views in
the reference's state-dict naming (core/model/src/model.rs:401-467, PyTorch ``[out, in]`` layout).
The same offsets index the gradient buffer, both AdamW moment buffers, the bf16 compute copy, the
round-start snapshot and the error-feedback buffer, so every per-parameter pass (AdamW, delta
extraction, compression, merge, broadcast) is a single kernel over one pointer range.

Within a layer the tensors that one GEMM consumes together are adjacent with no padding between
them: ``q_proj|k_proj|v_proj`` weights form the fused QKV weight ``[(nh+2nkv)d, H]``, their biases the
fused bias, and ``gate_proj|up_proj`` the fused ``[2F, H]`` gate/up weight. Every group starts on a
64-element boundary (256 B in fp32, 128 B in bf16: TMA needs 16 B).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Tuple

import torch

from ..config import ModelConfig

ALIGN = 64


@dataclass
class Entry:
    name: str
    shape: Tuple[int, ...]
    offset: int

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


def _ceil(x: int, a: int) -> int:
    return (x + a - 1) // a * a


class ParamLayout:
    def __init__(self, cfg: ModelConfig, tp_rank: int = 0, tp_size: int = 1):
        self.cfg = cfg
        self.tp_rank, self.tp_size = tp_rank, tp_size
        H, F, d = cfg.hidden_dim, cfg.ffn_hidden_dim, cfg.head_dim()
        nh, nkv = cfg.num_heads // tp_size, cfg.num_kv_heads // tp_size
        Ft = F // tp_size
        assert cfg.num_heads % tp_size == 0 and cfg.num_kv_heads % tp_size == 0 and F % tp_size == 0
        self.nh, self.nkv, self.d, self.F = nh, nkv, d, Ft
        self.entries: List[Entry] = []
        self.groups: Dict[str, Tuple[int, int]] = {}
        off = 0

        def group(gname: str, items):
            nonlocal off
            off = _ceil(off, ALIGN)
            start = off
            for name, shape in items:
                e = Entry(name, tuple(shape), off)
                self.entries.append(e)
                off += e.numel
            self.groups[gname] = (start, off)

        group("embedding", [("embedding.embedding.weight", (cfg.vocab_size, H))])
        group("output_scale", [("embedding.output_scale", (1,))])
        for i in range(cfg.num_layers):
            p = f"layers.{i}"
            group(f"{p}.attn_norm", [(f"{p}.attn_norm.weight", (H,))])
            group(f"{p}.qkv_w", [(f"{p}.attention.q_proj.weight", (nh * d, H)),
                                 (f"{p}.attention.k_proj.weight", (nkv * d, H)),
                                 (f"{p}.attention.v_proj.weight", (nkv * d, H))])
            if cfg.qkv_bias:
                group(f"{p}.qkv_b", [(f"{p}.attention.q_proj.bias", (nh * d,)),
                                     (f"{p}.attention.k_proj.bias", (nkv * d,)),
                                     (f"{p}.attention.v_proj.bias", (nkv * d,))])
            group(f"{p}.o_w", [(f"{p}.attention.o_proj.weight", (H, nh * d))])
            group(f"{p}.ffn_norm", [(f"{p}.ffn_norm.weight", (H,))])
            group(f"{p}.gu_w", [(f"{p}.ffn.gate_proj.weight", (Ft, H)), (f"{p}.ffn.up_proj.weight", (Ft, H))])
            group(f"{p}.down_w", [(f"{p}.ffn.down_proj.weight", (H, Ft))])
        group("final_norm", [("final_norm.weight", (H,))])
        self.total = _ceil(off, ALIGN)
        self.by_name = {e.name: e for e in self.entries}

    # ── views ──
    def views(self, flat: torch.Tensor) -> Dict[str, torch.Tensor]:
        return {e.name: flat[e.offset:e.offset + e.numel].view(e.shape) for e in self.entries}

    def view(self, flat: torch.Tensor, name: str) -> torch.Tensor:
        e = self.by_name[name]
        return flat[e.offset:e.offset + e.numel].view(e.shape)

    def group_view(self, flat: torch.Tensor, gname: str, shape=None) -> torch.Tensor:
        s, e = self.groups[gname]
        v = flat[s:e]
        return v.view(shape) if shape is not None else v

    def num_params(self) -> int:
        return sum(e.numel for e in self.entries)

    def shapes(self) -> Dict[str, List[int]]:
        return {e.name: list(e.shape) for e in self.entries}

    # ── state dict I/O ──
    def to_state_dict(self, flat: torch.Tensor) -> Dict[str, torch.Tensor]:
        return {k: v.detach().float().cpu().clone() for k, v in self.views(flat).items()}

    def load_state_dict(self, flat: torch.Tensor, sd: Dict[str, torch.Tensor]):
        views = self.views(flat)
        missing = [k for k in views if k not in sd]
        if missing:
            raise KeyError(f"state dict is missing {missing[:4]}{'...' if len(missing) > 4 else ''}")
        with torch.no_grad():
            for k, v in views.items():
                src = sd[k]
                if src.numel() != v.numel():
                    raise ValueError(f"{k}: expected {tuple(v.shape)} got {tuple(src.shape)}")
                v.copy_(src.reshape(v.shape).to(v.dtype))

    # ── optimizer chunk tables ──
    WINDOW = 1 << 31  # compressed payloads store kept indices relative to windows of this many elements

    def chunk_tables(self, device, chunk: int = 32768):
        """(cseg, cstart, cend) int32/int64 device tensors: one segment per named tensor, chunks of
        <= ``chunk`` elements with 4-aligned starts (the tail of a tensor may extend into padding). No chunk
        straddles a multiple of ``WINDOW``."""
        segs, starts, ends = [], [], []
        W = self.WINDOW
        for si, e in enumerate(self.entries):
            s, end = e.offset, e.offset + e.numel
            i = s
            while i < end:
                j = min(i + chunk, end, (i // W + 1) * W)
                segs.append(si)
                starts.append(i)
                ends.append(j)
                i = j
        t = lambda x, dt: torch.tensor(x, dtype=dt, device=device)
        return t(segs, torch.int32), t(starts, torch.int64), t(ends, torch.int64), len(self.entries)


def init_flat(layout: ParamLayout, std: float = 0.02, seed: int = 0, device="cpu") -> torch.Tensor:
    """Seeded N(0, std) weights, norm weights 1, biases 0, output_scale 1 (the benchmark init)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    flat = torch.zeros(layout.total, dtype=torch.float32)
    for e in layout.entries:
        v = flat[e.offset:e.offset + e.numel]
        if e.name.endswith("norm.weight") or e.name.endswith("output_scale"):
            v.fill_(1.0)
        elif e.name.endswith(".bias"):
            v.zero_()
        else:
            v.copy_(torch.randn(e.numel, generator=g) * std)
    return flat.to(device)
