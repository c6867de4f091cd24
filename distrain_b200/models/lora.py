"""Low-rank adapters (LoRA) trained on the CUDA engine with the base weights frozen.

The reference's post-training scripts offer ``--use-lora --lora-rank r --lora-alpha a``
(``scripts/run_sft.py:101-104,122-135``, ``scripts/run_dpo.py:59-60``); their trainer is not in its
repository. Here every projection of every block (the fused q|k|v, o, gate|up and down weights,
``[N, K]`` in the PyTorch layout, y = x W^T) gets W_eff = W + s B A with A ``[r, K]``, B ``[N, r]`` and
s = alpha / r (Hu et al., 2021); B starts at zero, A uniform in +-1/sqrt(K), so training starts from the
base model exactly.

How it runs on the fused engine: before a step the bf16 weights the GEMMs read are set to W_eff (the
fp32 master copy keeps the frozen W), the engine's forward and backward run unchanged and leave
dL/dW_eff in its gradient buffer, and two small products give the adapters' gradients,
dA = s B^T dW and dB = s dW A^T. The adapters have a flat fp32 buffer of their own with per-tensor
chunk tables, so the engine's AdamW kernel (per-tensor clipping, bias correction, decoupled weight
decay) updates them; the engine's AdamW moments for the frozen weights are released. The engine still
computes the full weight gradients, so a step costs what a full fine-tuning step costs; the saving is
the optimizer state and the size of what is trained and stored.
"""
from __future__ import annotations

import math
from typing import Dict, List, Tuple

import torch

from .. import ops
from .engine import (HP_B1 as _HP_B1, HP_B2 as _HP_B2, HP_CLIP_GLOBAL as _HP_CLIP_GLOBAL, HP_EPS as _HP_EPS,
                     HP_LR as _HP_LR, HP_MAXNORM as _HP_MAXNORM, HP_WD as _HP_WD, HP_ZERO_GRAD as _HP_ZERO_GRAD)

TARGETS = ("qkv_w", "o_w", "gu_w", "down_w")


class LoraAdapters:
    """Adapters for every block's projections of a ``TrainEngine`` (which must not be tensor-parallel)."""

    def __init__(self, eng, rank: int = 64, alpha: float = 128.0, lr: float = 1e-4, weight_decay: float = 0.0,
                 grad_clip_norm: float = 1.0, seed: int = 0, targets=TARGETS):
        if eng.tp is not None and eng.tp.size > 1:
            raise NotImplementedError("LoRA runs on engines without tensor parallelism")
        self.eng, self.r, self.s = eng, int(rank), float(alpha) / float(rank)
        L, dev = eng.layout, eng.device
        # (layer, name, frozen W, A, B, dA, dB) per adapted weight
        self.items: List[Tuple[int, str, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]] = []
        shapes = []
        for l in range(eng.cfg.num_layers):
            for name in targets:
                g = eng.gv[l][name]
                shapes.append((l, name, g.shape[0], g.shape[1]))
        # flat adapter buffer: per target A [r, K] then B [N, r], each padded to a multiple of 4 elements
        offs, off = [], 0
        for (_, _, N, K) in shapes:
            a, b = off, off + _pad4(self.r * K)
            off = b + _pad4(N * self.r)
            offs.append((a, b))
        self.total = off
        f32 = torch.float32
        self.p = torch.zeros(off, dtype=f32, device=dev)
        self.g = torch.zeros(off, dtype=f32, device=dev)
        self.m = torch.zeros(off, dtype=f32, device=dev)
        self.v = torch.zeros(off, dtype=f32, device=dev)
        gen = torch.Generator().manual_seed(seed)
        segs, starts, ends = [], [], []  # AdamW chunk tables: one segment (clipping unit) per A and per B
        nseg = 0
        for (l, name, N, K), (a, b) in zip(shapes, offs):
            A, B = self.p[a:a + self.r * K].view(self.r, K), self.p[b:b + N * self.r].view(N, self.r)
            gA, gB = self.g[a:a + self.r * K].view(self.r, K), self.g[b:b + N * self.r].view(N, self.r)
            A.copy_((torch.rand(self.r, K, generator=gen) * 2 - 1) / math.sqrt(K))
            W = L.group_view(eng.master, f"layers.{l}.{name}", (N, K))
            self.items.append((l, name, W, A, B, gA, gB))
            for lo, n in ((a, self.r * K), (b, N * self.r)):
                i = lo
                while i < lo + n:  # chunks of <= 32768 elements, 4-aligned starts
                    j = min(i + 32768, lo + n)
                    segs.append(nseg)
                    starts.append(i)
                    ends.append(j)
                    i = j
                nseg += 1
        t = lambda x, dt: torch.tensor(x, dtype=dt, device=dev)
        self.cseg, self.cstart, self.cend = t(segs, torch.int32), t(starts, torch.int64), t(ends, torch.int64)
        self.norms = torch.zeros(nseg, dtype=f32, device=dev)
        self.hp = torch.zeros(16, dtype=f32, device=dev)
        o = eng.optim
        hp = [0.0] * 16
        hp[_HP_B1], hp[_HP_B2], hp[_HP_EPS], hp[_HP_WD] = o.beta1, o.beta2, o.eps, weight_decay
        hp[_HP_MAXNORM], hp[_HP_CLIP_GLOBAL], hp[_HP_ZERO_GRAD] = grad_clip_norm, 0.0, 1.0
        hp[_HP_LR] = lr
        self.hp.copy_(torch.tensor(hp))
        # the frozen weights need no AdamW moments (the engine's own optimizer step is not used)
        eng.m = eng.v = None
        self.merge()

    def set_lr(self, lr: float):
        self.hp[_HP_LR:_HP_LR + 1].fill_(lr)

    def merge(self):
        """bf16 weights of the GEMMs <- W + s B A (the fp32 master keeps W)."""
        with torch.no_grad():
            for l, name, W, A, B, _, _ in self.items:
                self.eng.wv[l][name].copy_(torch.addmm(W, B, A, alpha=self.s))

    def step(self):
        """One training step of the adapters over the engine's micro-batches (tokens and loss weights set
        on the engine beforehand)."""
        eng = self.eng
        self.merge()
        for a in range(eng.A):
            eng.forward_backward(a, zero_grad=a == 0)
        with torch.no_grad():
            for l, name, _, A, B, gA, gB in self.items:
                dW = eng.gv[l][name]
                torch.mm(B.t(), dW, out=gA).mul_(self.s)
                torch.mm(dW, A.t(), out=gB).mul_(self.s)
        ops.adamw_step(self.p, self.g, self.m, self.v, None, self.cseg, self.cstart, self.cend, self.norms, self.hp,
                       eng.loss)
        self.merge()

    def merged_state_dict(self) -> Dict[str, torch.Tensor]:
        """The full model with the adapters folded in (fp32, the checkpoint layout)."""
        flat = self.eng.master.clone()
        L = self.eng.layout
        with torch.no_grad():
            for l, name, W, A, B, _, _ in self.items:
                L.group_view(flat, f"layers.{l}.{name}", tuple(W.shape)).add_(B @ A, alpha=self.s)
        return L.to_state_dict(flat)

    def adapter_state_dict(self) -> Dict[str, torch.Tensor]:
        out = {}
        for l, name, _, A, B, _, _ in self.items:
            out[f"layers.{l}.{name}.lora_A"] = A.detach().float().cpu().clone()
            out[f"layers.{l}.{name}.lora_B"] = B.detach().float().cpu().clone()
        return out


def _pad4(n: int) -> int:
    return (n + 3) // 4 * 4
