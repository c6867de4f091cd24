"""Plain-PyTorch fp32 restatement of the reference transformer (the numerics oracle and the CPU path).

Follows core/model/src/model.rs op by op:
* RMSNorm ``x * rsqrt(mean(x^2) + eps) * w`` (:51-59)
* q/k/v Linear with bias, o_proj without (:193-204); RoPE rotate-half with fp32 tables
  ``freq_i = 1/theta^(2i/d)`` (:66-122)
* GQA by repeating each kv head over its group (:127-138); scores ``q k^T / sqrt(d)`` plus an additive
  causal mask of -1e4 (:142-166, :246-256); softmax; ``P V``
* SwiGLU ``down(silu(gate x) * up x)`` (:292-296); pre-norm residual blocks (:366-375)
* final norm, tied head ``(h * output_scale) E^T`` (:323-339)
* loss ``-mean(log_softmax(logits)[target])`` on ``tokens[:, :-1] -> tokens[:, 1:]`` (:783-812)

``mask_value=None`` swaps the -1e4 additive mask for an exact -inf mask (what a flash kernel computes);
the two agree to far below fp32 resolution for any realistic score range.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn.functional as Fn

from ..config import ModelConfig


def rope_tables(cfg: ModelConfig, seq: int, device="cpu"):
    """fp32 cos/sin [seq, d/2] computed exactly like the reference (fp32 pow, fp32 outer product)."""
    d = cfg.head_dim()
    half = d // 2
    i = torch.arange(half, dtype=torch.float32)
    theta = torch.tensor(cfg.rope_theta, dtype=torch.float32)
    freqs = 1.0 / torch.pow(theta, 2.0 * i / d)
    t = torch.arange(seq, dtype=torch.float32)
    ang = t[:, None] * freqs[None, :]
    return torch.cos(ang).to(device), torch.sin(ang).to(device)


def rms_norm(x, w, eps):
    var = x.pow(2).mean(-1, keepdim=True)
    return x * (var + eps).sqrt().reciprocal() * w


def apply_rope(x, cos, sin):
    # x: [B, T, heads, d]
    half = x.shape[-1] // 2
    c = cos[None, :, None, :]
    s = sin[None, :, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


def forward_hidden(p: Dict[str, torch.Tensor], cfg: ModelConfig, ids: torch.Tensor,
                   mask_value: Optional[float] = -1e4) -> torch.Tensor:
    B, T = ids.shape
    d, nh, nkv = cfg.head_dim(), cfg.num_heads, cfg.num_kv_heads
    groups = nh // nkv
    cos, sin = rope_tables(cfg, T, ids.device)
    h = p["embedding.embedding.weight"][ids]
    causal = torch.triu(torch.ones(T, T, dtype=torch.bool, device=ids.device), diagonal=1)
    for i in range(cfg.num_layers):
        pre = f"layers.{i}"
        x = rms_norm(h, p[f"{pre}.attn_norm.weight"], cfg.norm_eps)

        def lin(name, inp, bias=True):
            y = inp @ p[f"{pre}.attention.{name}.weight"].t()
            b = p.get(f"{pre}.attention.{name}.bias")
            return y + b if (bias and b is not None) else y

        q = lin("q_proj", x).view(B, T, nh, d)
        k = lin("k_proj", x).view(B, T, nkv, d)
        v = lin("v_proj", x).view(B, T, nkv, d)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        k = k.repeat_interleave(groups, dim=2)
        v = v.repeat_interleave(groups, dim=2)
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        s = (q @ k.transpose(-1, -2)) / (d ** 0.5)
        if mask_value is None:
            s = s.masked_fill(causal, float("-inf"))
        else:
            s = s + causal.to(s.dtype) * mask_value
        a = torch.softmax(s, dim=-1) @ v
        a = a.transpose(1, 2).reshape(B, T, nh * d)
        h = h + a @ p[f"{pre}.attention.o_proj.weight"].t()
        x = rms_norm(h, p[f"{pre}.ffn_norm.weight"], cfg.norm_eps)
        g = x @ p[f"{pre}.ffn.gate_proj.weight"].t()
        u = x @ p[f"{pre}.ffn.up_proj.weight"].t()
        h = h + (Fn.silu(g) * u) @ p[f"{pre}.ffn.down_proj.weight"].t()
    return rms_norm(h, p["final_norm.weight"], cfg.norm_eps)


def logits_fn(p, cfg, ids, mask_value=-1e4):
    h = forward_hidden(p, cfg, ids, mask_value)
    return (h * p["embedding.output_scale"]) @ p["embedding.embedding.weight"].t()


def lm_loss(p: Dict[str, torch.Tensor], cfg: ModelConfig, tokens: torch.Tensor, mask_value=-1e4) -> torch.Tensor:
    """Reference ``compute_lm_loss``: predict tokens[:, 1:] from tokens[:, :-1]."""
    inp, tgt = tokens[:, :-1], tokens[:, 1:]
    z = logits_fn(p, cfg, inp, mask_value)
    lp = torch.log_softmax(z.reshape(-1, z.shape[-1]).float(), dim=-1)
    return -lp.gather(1, tgt.reshape(-1, 1).long()).mean()


class AdamWRef:
    """fp32 AdamW with per-tensor gradient-norm clipping (the reference inner optimiser's semantics)."""

    def __init__(self, params: Dict[str, torch.Tensor], lr=3e-4, betas=(0.9, 0.999), eps=1e-5, weight_decay=0.1,
                 clip=1.0, clip_global=False):
        self.p = params
        self.lr, self.b1, self.b2, self.eps, self.wd, self.clip = lr, betas[0], betas[1], eps, weight_decay, clip
        self.clip_global = clip_global
        self.m = {k: torch.zeros_like(v) for k, v in params.items()}
        self.v = {k: torch.zeros_like(v) for k, v in params.items()}
        self.t = 0

    @torch.no_grad()
    def step(self, lr: Optional[float] = None):
        lr = self.lr if lr is None else lr
        self.t += 1
        bc1, bc2 = 1 - self.b1 ** self.t, 1 - self.b2 ** self.t
        if self.clip_global and self.clip > 0:
            tot = torch.sqrt(sum((q.grad.double() ** 2).sum() for q in self.p.values() if q.grad is not None))
            gcoef = min(1.0, self.clip / (float(tot) + 1e-6))
        for k, q in self.p.items():
            if q.grad is None:
                continue
            g = q.grad
            if self.clip > 0:
                coef = gcoef if self.clip_global else min(1.0, self.clip / (float(g.norm()) + 1e-6))
                g = g * coef
            self.m[k].mul_(self.b1).add_(g, alpha=1 - self.b1)
            self.v[k].mul_(self.b2).addcmul_(g, g, value=1 - self.b2)
            upd = (self.m[k] / bc1) / (torch.sqrt(self.v[k] / bc2) + self.eps)
            q.mul_(1 - lr * self.wd).sub_(upd, alpha=lr)
            q.grad = None
