"""Node training engine: explicit forward + backward + AdamW over flat buffers, graph-capturable.

One ``TrainEngine`` owns, for one model replica on one GPU:

* ``master`` fp32 flat parameters, ``p16`` bf16 compute copy, ``grad`` fp32, AdamW ``m``/``v``;
* every activation buffer of one micro-batch geometry (B sequences of S tokens), allocated once;
* a device hyper-parameter block (lr, betas, eps, wd, step, bias corrections) and a device loss
  scalar, so ``step()`` issues no host synchronisation and can be replayed from a CUDA graph.

Per step (all on the current stream):
  embed+RMSNorm -> L x [QKV GEMM with bias+RoPE epilogue, flash attention, O GEMM, add+RMSNorm, gate|up
  GEMM with SwiGLU epilogue, down GEMM, add+RMSNorm] -> chunked tied LM head GEMM with fp32 softmax
  statistics in its epilogue + cross-entropy (loss from fp32, in-place dlogits)
  -> backward in reverse (dgrad/wgrad tcgen05 GEMMs, norm/rope/swiglu/attention backward,
  embedding scatter-add) -> per-tensor clip + AdamW (also refreshes ``p16``).

The step mirrors the reference's continuous-loop step (node/cli/src/continuous.rs:598-637): loss on
tokens[:, :-1] -> tokens[:, 1:], a NaN loss skips the optimiser update (decided on the device).

Gradient accumulation (``grad_accum`` = A > 1): one step takes A micro-batches of B sequences
(``ids`` is [A*B, S]); forward + backward run once per micro-batch on the same activation buffers, the
weight-gradient GEMMs accumulate into the fp32 gradients, the loss is the mean over all A*B*T tokens,
and clipping + AdamW run once per step. This is the accumulation the reference's trainer intends
(node/cli/src/trainer.rs:592-630), where the optimiser instead steps after every micro-batch.
Gradients are cleared by the AdamW kernel after it has read them (also on a skipped step), so no
separate zeroing pass runs inside a step.

Options: ``tp`` (a ``parallel.tensor_parallel.TensorParallel``) runs this replica split over a
tensor-parallel group (local heads / FFN rows; all-reduces after the row-parallel GEMMs in the forward
and the column-parallel data-gradient GEMMs in the backward; group-summed clip norms). ``act_ckpt``
keeps only each block's input residual and recomputes the block's forward (norm, QKV, RoPE, attention,
o_proj, norm, gate|up, SwiGLU) right before its backward, with one set of block buffers.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import ops
from ..ops import attention as attn_ops
from ..config import ModelConfig, OptimConfig
from .params import ParamLayout, init_flat
from .oracle import rope_tables

HP_LR, HP_B1, HP_B2, HP_EPS, HP_WD, HP_BC1, HP_BC2, HP_MAXNORM, HP_CLIP_GLOBAL, HP_STEP, HP_DO_UPDATE, \
    HP_ZERO_GRAD = range(12)


class TrainEngine:
    def __init__(self, cfg: ModelConfig, batch: int, seq_len: int, optim: Optional[OptimConfig] = None,
                 device="cuda", flat_init: Optional[torch.Tensor] = None, seed: int = 0, init_std: float = 0.02,
                 lm_chunk_rows: int = 32768, attn_impl: str = "dt", tp=None, act_ckpt: bool = False,
                 grad_accum: int = 1, loss_weights: bool = False, inference: bool = False,
                 weights_from: Optional["TrainEngine"] = None):
        """``inference``: forward-only engine (``forward_loss``): no gradients, optimizer state or
        backward scratch, and one set of per-block activation buffers shared by all blocks.
        ``weights_from``: an engine of the same model whose fp32 and bf16 weights this one uses (not
        copies; ``flat_init`` is ignored), e.g. forward-only engines of several sequence lengths."""
        self.cfg = cfg
        self.inference = inference
        self.tp = tp
        self.act_ckpt = act_ckpt
        tp_rank, tp_size = (tp.rank, tp.size) if tp is not None else (0, 1)
        self.optim = optim or OptimConfig()
        self.device = torch.device(device)
        self.B, self.S = batch, seq_len
        self.A = max(int(grad_accum), 1)
        self.T = seq_len - 1
        self.M = self.B * self.T
        self.attn_impl = attn_impl
        L = self.layout = ParamLayout(cfg, tp_rank, tp_size)
        # local (per tensor-parallel rank) head counts and FFN width
        H, F, d, nh, nkv, V = cfg.hidden_dim, L.F, cfg.head_dim(), L.nh, L.nkv, cfg.vocab_size
        self.H, self.F, self.d, self.nh, self.nkv, self.V = H, F, d, nh, nkv, V
        self.W = (nh + 2 * nkv) * d
        dev = self.device
        f32, bf16 = torch.float32, torch.bfloat16
        n = L.total
        # ── parameters / optimizer state ──
        if weights_from is not None:
            if weights_from.layout.total != n or weights_from.device != dev:
                raise ValueError("weights_from: an engine of another model layout or device")
            self.master, self.p16 = weights_from.master, weights_from.p16
        else:
            self.master = torch.zeros(n, dtype=f32, device=dev)
            self.p16 = torch.zeros(n, dtype=bf16, device=dev)
        self.grad = None if inference else torch.zeros(n, dtype=f32, device=dev)
        self.m = None if inference else torch.zeros(n, dtype=f32, device=dev)
        self.v = None if inference else torch.zeros(n, dtype=f32, device=dev)
        self.cseg, self.cstart, self.cend, self.nseg = L.chunk_tables(dev)
        self.norms = torch.zeros(self.nseg, dtype=f32, device=dev)
        self.hp = torch.zeros(16, dtype=f32, device=dev)
        self._hp_host = torch.zeros(16, dtype=f32).pin_memory() if dev.type == "cuda" else torch.zeros(16)
        # ── inputs / outputs ──
        self.ids = torch.zeros(self.A * batch, seq_len, dtype=torch.int32, device=dev)
        self.loss = torch.zeros(4, dtype=f32, device=dev)  # [mean loss, nonfinite flag, -, -]
        cos, sin = rope_tables(cfg, self.T)
        self.cos, self.sin = cos.to(dev).contiguous(), sin.to(dev).contiguous()
        # ── activations (saved for backward) ──
        M, Lr = self.M, cfg.num_layers
        Tp = attn_ops.lse_stride(self.T)
        # with activation checkpointing (or forward only) every block shares one set of buffers (index 0)
        nb = 1 if (act_ckpt or inference) else Lr

        def per_block(make):
            bufs = [make() for _ in range(nb)]
            return bufs * Lr if nb == 1 else bufs
        self.resid_in = [torch.empty(M, H, dtype=f32, device=dev) for _ in range(Lr)]
        self.resid_mid = per_block(lambda: torch.empty(M, H, dtype=f32, device=dev))
        self.rstd1 = per_block(lambda: torch.empty(M, dtype=f32, device=dev))
        self.rstd2 = per_block(lambda: torch.empty(M, dtype=f32, device=dev))
        self.xn1 = per_block(lambda: torch.empty(M, H, dtype=bf16, device=dev))
        self.xn2 = per_block(lambda: torch.empty(M, H, dtype=bf16, device=dev))
        self.qkv = per_block(lambda: torch.empty(M, self.W, dtype=bf16, device=dev))
        self.attn = per_block(lambda: torch.empty(M, nh * d, dtype=bf16, device=dev))
        self.lse = per_block(lambda: torch.empty(batch, nh, Tp, dtype=f32, device=dev))
        self.gu = per_block(lambda: torch.empty(M, 2 * F, dtype=bf16, device=dev))
        self.hact = per_block(lambda: torch.empty(M, F, dtype=bf16, device=dev))
        self.resid_fin = torch.empty(M, H, dtype=f32, device=dev)
        self.rstd_f = torch.empty(M, dtype=f32, device=dev)
        self.xs = torch.empty(M, H, dtype=bf16, device=dev)
        self.lm_chunk = min(lm_chunk_rows, M)
        self.logits = torch.empty(self.lm_chunk, V, dtype=bf16, device=dev)
        # softmax statistics of the LM-head GEMM (fp32 max / sum exp per row and half tile) and the
        # fp32 target logits: the loss and its log-sum-exp come from the fp32 accumulators
        self.lse_part = torch.empty(ops.lse_parts(self.lm_chunk, V) * 2, dtype=f32, device=dev)
        self.tgt_logit = torch.empty(self.lm_chunk, dtype=f32, device=dev)
        self.loss_rows = torch.empty(self.A * M, dtype=f32, device=dev)
        # per-row loss weights of the step (fine-tuning masks, preference coefficients): the loss is
        # sum_r w_r * ce_r over all micro-batches and each row's gradient is scaled by w_r, so the weights
        # carry the normalisation. Without them the loss is the mean over rows.
        self.loss_w = torch.zeros(self.A * M, dtype=f32, device=dev) if loss_weights else None
        # ── backward scratch ──
        bwd_empty = (lambda *shape, dtype=f32: torch.empty(*shape, dtype=dtype, device=dev)) if not inference \
            else (lambda *shape, dtype=f32: None)
        self.br = torch.empty(M, H, dtype=bf16, device=dev)  # also the forward's row-parallel GEMM output
        self.dresid = bwd_empty(M, H)
        self.g16 = bwd_empty(M, H, dtype=bf16)
        self.dxs = bwd_empty(M, H, dtype=bf16)
        # SwiGLU fused into the gate/up GEMM's epilogue when F is a multiple of 64 (else a separate
        # activation kernel). The backward's fused form (dh kept in the down-projection data-gradient
        # GEMM, whose epilogue reads the saved gate / up tile by TMA) measured 0.260 ms per tiny layer
        # against 0.214 ms for the plain GEMM + the bandwidth-bound activation kernel: a 128-row tile's
        # 64 KB of gate / up cannot be double-buffered beside the operand ring. It stays selectable.
        self.fused_swiglu = F % 64 == 0
        self.fused_swiglu_bwd = False
        self.dh = None if self.fused_swiglu_bwd else bwd_empty(M, F, dtype=bf16)
        self.dgu = bwd_empty(M, 2 * F, dtype=bf16)
        self.dattn = bwd_empty(M, nh * d, dtype=bf16)
        self.dqkv = bwd_empty(M, self.W, dtype=bf16)
        self.dq_acc = bwd_empty(M, nh * d)
        self.delta = bwd_empty(batch, nh, Tp)
        # per-block column sums of the QKV bias gradient (RoPE backward)
        self.rope_part = (bwd_empty(ops.rope_bwd_scratch(M, nh, nkv, d))
                          if cfg.qkv_bias and dev.type == "cuda" else None)
        # dS^T tiles of one layer's attention backward (tcgen05 path): dQ is formed from them by a GEMM-like
        # kernel instead of a second pass over S, P and dP
        self.ds_buf = None
        if (not inference and attn_ops.bwd_kernel_for(d, attn_impl) == "tc" and d in (64, 128)
                and dev.type == "cuda"):
            self.ds_buf = torch.empty(attn_ops.ds_bytes(batch, self.T, nh), dtype=torch.uint8, device=dev)
        if tp is not None:
            from ..parallel.tensor_parallel import norm_weights
            self.norm_w = norm_weights(L, dev)
        # ── named views ──
        self._bind_views()
        if weights_from is not None:
            self._write_hp(self.optim.lr)
        else:
            if flat_init is None:
                if tp is not None and tp.size > 1:
                    from ..parallel.tensor_parallel import init_flat_tp
                    flat_init = init_flat_tp(L, init_std, seed, device=dev)
                else:
                    flat_init = init_flat(L, init_std, seed)
            self.load_flat(flat_init)
        self.graph = None
        self.kernels_per_step = 0

    # ───────────────────────── parameter views ─────────────────────────
    def _bind_views(self):
        L, cfg = self.layout, self.cfg
        H, F, W, nh, d = self.H, self.F, self.W, self.nh, self.d

        def trip(buf, prefix_dtype_views):
            return prefix_dtype_views

        self.pv, self.gv, self.wv = [], [], []
        for i in range(cfg.num_layers):
            p = f"layers.{i}"
            ent = {
                "attn_norm": L.view(self.master, f"{p}.attn_norm.weight"),
                "ffn_norm": L.view(self.master, f"{p}.ffn_norm.weight"),
                "qkv_b": L.group_view(self.master, f"{p}.qkv_b") if cfg.qkv_bias else None,
            }
            gr = None if self.grad is None else {
                "attn_norm": L.view(self.grad, f"{p}.attn_norm.weight"),
                "ffn_norm": L.view(self.grad, f"{p}.ffn_norm.weight"),
                "qkv_b": L.group_view(self.grad, f"{p}.qkv_b") if cfg.qkv_bias else None,
                "qkv_w": L.group_view(self.grad, f"{p}.qkv_w", (W, H)),
                "o_w": L.group_view(self.grad, f"{p}.o_w", (H, nh * d)),
                "gu_w": L.group_view(self.grad, f"{p}.gu_w", (2 * F, H)),
                "down_w": L.group_view(self.grad, f"{p}.down_w", (H, F)),
            }
            w16 = {
                "qkv_w": L.group_view(self.p16, f"{p}.qkv_w", (W, H)),
                "o_w": L.group_view(self.p16, f"{p}.o_w", (H, nh * d)),
                "gu_w": L.group_view(self.p16, f"{p}.gu_w", (2 * F, H)),
                "down_w": L.group_view(self.p16, f"{p}.down_w", (H, F)),
            }
            self.pv.append(ent)
            self.gv.append(gr)
            self.wv.append(w16)
        self.E = L.view(self.master, "embedding.embedding.weight")
        self.E16 = L.view(self.p16, "embedding.embedding.weight")
        self.oscale = L.view(self.master, "embedding.output_scale")
        self.fnorm = L.view(self.master, "final_norm.weight")
        if self.grad is not None:
            self.gE = L.view(self.grad, "embedding.embedding.weight")
            self.g_oscale = L.view(self.grad, "embedding.output_scale")
            self.g_fnorm = L.view(self.grad, "final_norm.weight")

    # ───────────────────────── state management ─────────────────────────
    def load_flat(self, flat: torch.Tensor, reset_optimizer: bool = True):
        """Replace master weights (e.g. a new global checkpoint) and optionally reset AdamW state."""
        with torch.no_grad():
            self.master.copy_(flat.to(self.device, non_blocking=True))
            ops.cast_bf16(self.master, self.p16)
            if reset_optimizer and self.m is not None:
                self.m.zero_()
                self.v.zero_()
                self.hp.zero_()
                self._write_hp(self.optim.lr)

    def _write_hp(self, lr: float):
        o = self.optim
        h = self._hp_host
        h[HP_LR] = lr
        h[HP_B1], h[HP_B2], h[HP_EPS], h[HP_WD] = o.beta1, o.beta2, o.eps, o.weight_decay
        h[HP_MAXNORM] = o.grad_clip_norm
        h[HP_CLIP_GLOBAL] = 1.0 if o.clip_global else 0.0
        h[HP_ZERO_GRAD] = 1.0
        # copy only the configuration slots; step/bias-correction/skip slots are device-owned
        self.hp[:HP_BC1].copy_(h[:HP_BC1], non_blocking=True)
        self.hp[HP_MAXNORM:HP_STEP].copy_(h[HP_MAXNORM:HP_STEP], non_blocking=True)
        self.hp[HP_ZERO_GRAD:HP_ZERO_GRAD + 1].copy_(h[HP_ZERO_GRAD:HP_ZERO_GRAD + 1], non_blocking=True)

    def set_lr(self, lr: float):
        self._write_hp(lr)

    def set_tokens(self, tokens: torch.Tensor):
        """[A*B, S] int32 token ids of one step (A micro-batches of B sequences)."""
        self.ids.copy_(tokens, non_blocking=True)

    def set_loss_weights(self, w: torch.Tensor):
        """Per-row loss weights of one step: [A*B, S-1] (weight of predicting token t+1 of a sequence) or
        flat [A*M]. Needs an engine built with ``loss_weights=True``."""
        if self.loss_w is None:
            raise RuntimeError("engine built without loss_weights=True")
        self.loss_w.copy_(w.reshape(-1).to(torch.float32), non_blocking=True)

    # ───────────────────────── the step ─────────────────────────
    def forward_backward(self, micro: int = 0, zero_grad: bool = True):
        """Forward + backward of micro-batch ``micro`` (rows [micro*B, (micro+1)*B) of ``ids``), adding its
        gradients into ``grad`` (cleared first when ``zero_grad``); the loss of the step is reduced after
        the last micro-batch."""
        if self.inference:
            raise RuntimeError("forward_backward on a forward-only (inference) engine")
        M, Lr = self.M, self.cfg.num_layers
        if self._tp_active() and self.tp.fused:
            self.tp.begin_step(4 * Lr + ((Lr - 1) if self.act_ckpt else 0))
        if zero_grad:
            self.grad.zero_()
        ids = self.ids[micro * self.B:(micro + 1) * self.B]
        self._forward(ids)
        self._lm_head_loss(micro, ids, backward=True)
        if micro == self.A - 1:
            if self.loss_w is None:
                ops.loss_reduce(self.loss_rows, self.A * M, 1.0 / (M * self.A), self.loss)
            else:
                ops.loss_reduce(self.loss_rows, self.A * M, 1.0, self.loss, w=self.loss_w)
        self._backward(ids)

    def forward_loss(self, micro: int = 0) -> torch.Tensor:
        """Forward only: the unweighted cross-entropy of every row of micro-batch ``micro`` ([B*(S-1)] fp32
        view, predicting token t+1 of each sequence), e.g. for sequence log-probabilities. Parameters,
        gradients and the step's loss are left alone."""
        if self._tp_active():
            raise NotImplementedError("forward_loss runs on engines without tensor parallelism")
        ids = self.ids[micro * self.B:(micro + 1) * self.B]
        self._forward(ids)
        self._lm_head_loss(micro, ids, backward=False)
        return self.loss_rows[micro * self.M:(micro + 1) * self.M]

    def forward_hidden(self, micro: int = 0) -> torch.Tensor:
        """Forward only, up to the LM head's input: [B*(S-1), H] bf16 rows (final RMSNorm times the output
        scale), row b*(S-1) + t for position t of sequence b; logits = rows @ E^T (tied embedding)."""
        if self._tp_active():
            raise NotImplementedError("forward_hidden runs on engines without tensor parallelism")
        self._forward(self.ids[micro * self.B:(micro + 1) * self.B])
        return self.xs

    def _forward(self, ids):
        cfg = self.cfg
        M, H, T, S, d, nh, nkv = self.M, self.H, self.T, self.S, self.d, self.nh, self.nkv
        eps = cfg.norm_eps
        Lr = cfg.num_layers
        ops.add_rmsnorm_fwd(emb=self.E, ids=ids, T=T, S=S, w=self.pv[0]["attn_norm"], out_resid=self.resid_in[0],
                            y=self.xn1[0], rstd=self.rstd1[0], eps=eps, M=M, H=H)
        for l in range(Lr):
            pv, wv = self.pv[l], self.wv[l]
            self._qkv_rope(l)
            attn_ops.attention_fwd(self.qkv[l], self.attn[l], self.lse[l], B=self.B, T=T, nh=nh, nkv=nkv, d=d,
                                   impl=self.attn_impl)
            self._row_parallel_add_norm(self.attn[l], wv["o_w"], x=self.resid_in[l], w=pv["ffn_norm"],
                                        out_resid=self.resid_mid[l], y=self.xn2[l], rstd=self.rstd2[l])
            self._gate_up_swiglu(l)
            if l + 1 < Lr:
                self._row_parallel_add_norm(self.hact[l], wv["down_w"], x=self.resid_mid[l],
                                            w=self.pv[l + 1]["attn_norm"], out_resid=self.resid_in[l + 1],
                                            y=self.xn1[l + 1], rstd=self.rstd1[l + 1])
            else:
                self._row_parallel_add_norm(self.hact[l], wv["down_w"], x=self.resid_mid[l], w=self.fnorm,
                                            scale=self.oscale, out_resid=self.resid_fin, y=self.xs, rstd=self.rstd_f)

    def _lm_head_loss(self, micro: int, ids, backward: bool):
        """Tied LM head + cross-entropy, chunked over rows; the head's backward is fused per chunk."""
        M, H, T, S, V = self.M, self.H, self.T, self.S, self.V
        loss_rows = self.loss_rows[micro * M:(micro + 1) * M]
        row_w = None if self.loss_w is None else self.loss_w[micro * M:(micro + 1) * M]
        scale = 1.0 / (M * self.A) if row_w is None else 1.0
        for r0 in range(0, M, self.lm_chunk):
            rows = min(self.lm_chunk, M - r0)
            xs_c = self.xs[r0:r0 + rows]
            lg = self.logits[:rows]
            part = self.lse_part[:2 * ops.lse_parts(rows, V)]
            ops.gemm_logits_lse(xs_c, self.E16, lg, part, self.tgt_logit, ids, rows=rows, V=V, K=H, T=T, S=S, r0=r0)
            ops.ce_lse_bwd(lg, part, self.tgt_logit, ids, loss_rows[r0:r0 + rows], rows=rows, V=V, T=T, S=S, r0=r0,
                           grad_scale=scale, row_w=row_w)
            if not backward:
                continue
            ops.gemm(lg, self.E16, self.dxs[r0:r0 + rows], M=rows, N=H, K=V, b_mn=True, ldb=H)
            ops.gemm(lg, xs_c, self.gE, M=V, N=H, K=rows, a_mn=True, lda=V, b_mn=True, ldb=H, ldc=H,
                     epi=ops.EPI_F32_ATOMIC)

    def _backward(self, ids):
        M, H, F, T, S, d, nh, nkv = self.M, self.H, self.F, self.T, self.S, self.d, self.nh, self.nkv
        Lr = self.cfg.num_layers
        ops.rmsnorm_bwd(dy=self.dxs, x=self.resid_fin, rstd=self.rstd_f, w=self.fnorm, scale=self.oscale,
                        dresid_out=self.dresid, dresid16=self.g16, dw=self.g_fnorm, dscale=self.g_oscale, M=M, H=H)
        for l in reversed(range(Lr)):
            pv, wv, gv = self.pv[l], self.wv[l], self.gv[l]
            if self.act_ckpt and l + 1 < Lr:  # the last block's buffers are still live from the forward
                self._recompute_block(l)
            # FFN block
            if self.fused_swiglu_bwd:  # dh stays in the GEMM: its epilogue writes the SwiGLU backward
                ops.gemm_swiglu_bwd(self.g16, wv["down_w"], self.gu[l], self.dgu)
                ops.linear_wgrad(self.g16, self.hact[l], gv["down_w"])
            else:
                ops.linear_dgrad(self.g16, wv["down_w"], self.dh)
                ops.linear_wgrad(self.g16, self.hact[l], gv["down_w"])
                ops.swiglu_bwd(self.dh, self.gu[l], self.dgu, M=M, F=F)
            self._col_parallel_dgrad_norm_bwd(
                self.dgu, wv["gu_w"], lambda: ops.linear_wgrad(self.dgu, self.xn2[l], gv["gu_w"]),
                x=self.resid_mid[l], rstd=self.rstd2[l], w=pv["ffn_norm"], dresid_in=self.dresid,
                dresid_out=self.dresid, dresid16=self.g16, dw=gv["ffn_norm"])
            # attention block
            ops.linear_dgrad(self.g16, wv["o_w"], self.dattn)
            ops.linear_wgrad(self.g16, self.attn[l], gv["o_w"])
            attn_ops.attention_bwd(self.qkv[l], self.attn[l], self.dattn, self.lse[l], self.dqkv, self.dq_acc,
                                   self.delta, B=self.B, T=T, nh=nh, nkv=nkv, d=d, impl=self.attn_impl,
                                   ds_buf=self.ds_buf)
            ops.rope_bwd(self.dqkv, gv["qkv_b"], self.cos, self.sin, M=M, T=T, nh=nh, nkv=nkv, d=d,
                         part=self.rope_part)
            self._col_parallel_dgrad_norm_bwd(
                self.dqkv, wv["qkv_w"], lambda: ops.linear_wgrad(self.dqkv, self.xn1[l], gv["qkv_w"]),
                x=self.resid_in[l], rstd=self.rstd1[l], w=pv["attn_norm"], dresid_in=self.dresid,
                dresid_out=self.dresid, dresid16=self.g16 if l > 0 else None, dw=gv["attn_norm"])
        ops.embedding_bwd(self.dresid, ids, self.gE, T=T, S=S, M=M, H=H)

    def _qkv_rope(self, l: int):
        """qkv = rope(xn1 @ qkv_w^T + qkv_b): bias and rotation in the GEMM's epilogue for head dims 64 /
        128, else a separate in-place pass."""
        T, d, nh, nkv = self.T, self.d, self.nh, self.nkv
        if d in (64, 128):
            ops.gemm_qkv_rope(self.xn1[l], self.wv[l]["qkv_w"], self.pv[l]["qkv_b"], self.cos, self.sin, self.qkv[l],
                              T=T, d=d, rot_cols=(nh + nkv) * d)
        else:
            ops.linear_fwd(self.xn1[l], self.wv[l]["qkv_w"], self.qkv[l])
            ops.rope_fwd(self.qkv[l], self.pv[l]["qkv_b"], self.cos, self.sin, M=self.M, T=T, nh=nh, nkv=nkv, d=d)

    def _gate_up_swiglu(self, l: int):
        """gu = xn2 @ gu_w^T and h = silu(gate) * up: one GEMM with the activation in its epilogue."""
        if self.fused_swiglu:
            ops.gemm_swiglu_fwd(self.xn2[l], self.wv[l]["gu_w"], self.gu[l], self.hact[l])
        else:
            ops.linear_fwd(self.xn2[l], self.wv[l]["gu_w"], self.gu[l])
            ops.swiglu_fwd(self.gu[l], self.hact[l], M=self.M, F=self.F)

    def _tp_active(self) -> bool:
        return self.tp is not None and self.tp.size > 1

    def _row_parallel_add_norm(self, a, w16, *, x, w, y, rstd, out_resid=None, scale=None):
        """br = a @ w16^T (summed over the tensor-parallel group), then resid = x + br, y = rmsnorm(resid)."""
        M, H, eps = self.M, self.H, self.cfg.norm_eps
        if self._tp_active() and self.tp.fused:
            tp = self.tp
            slot = tp.next_slot()
            ops.linear_peer(a, w16, self.br, tp.peer_recv_ptr(slot), tp.peer_arrivals, tp.done_ctas)
            ops.add_rmsnorm_fwd_tp(x=x, br=self.br, br2=tp.recv(slot), w=w, scale=scale, out_resid=out_resid, y=y,
                                   rstd=rstd, eps=eps, M=M, H=H, arrivals=tp.arrivals, consumed=tp.consumed,
                                   done_blocks=tp.done_blocks)
            return
        ops.linear_fwd(a, w16, self.br)
        if self._tp_active():
            self.tp.allreduce_(self.br)
        ops.add_rmsnorm_fwd(x=x, br=self.br, w=w, scale=scale, out_resid=out_resid, y=y, rstd=rstd, eps=eps, M=M,
                            H=H)

    def _col_parallel_dgrad_norm_bwd(self, dy, w16, between, *, x, rstd, w, dresid_in, dresid_out, dresid16, dw):
        """br = dy @ w16 (summed over the group), ``between()`` (independent work that overlaps the
        exchange), then the RMSNorm backward taking br as its incoming gradient."""
        M, H = self.M, self.H
        if self._tp_active() and self.tp.fused:
            tp = self.tp
            slot = tp.next_slot()
            ops.linear_peer(dy, w16, self.br, tp.peer_recv_ptr(slot), tp.peer_arrivals, tp.done_ctas, dgrad=True)
            between()
            ops.rmsnorm_bwd_tp(dy=self.br, dy2=tp.recv(slot), x=x, rstd=rstd, w=w, dresid_in=dresid_in,
                               dresid_out=dresid_out, dresid16=dresid16, dw=dw, M=M, H=H, arrivals=tp.arrivals,
                               consumed=tp.consumed, done_blocks=tp.done_blocks)
            return
        ops.linear_dgrad(dy, w16, self.br)
        if self._tp_active():
            self.tp.allreduce_(self.br)
        between()
        ops.rmsnorm_bwd(dy=self.br, x=x, rstd=rstd, w=w, dresid_in=dresid_in, dresid_out=dresid_out,
                        dresid16=dresid16, dw=dw, M=M, H=H)

    def _recompute_block(self, l: int):
        """Forward of block l from its saved input residual, into the shared block buffers."""
        cfg = self.cfg
        M, H, F, T, d, nh, nkv = self.M, self.H, self.F, self.T, self.d, self.nh, self.nkv
        pv, wv = self.pv[l], self.wv[l]
        eps = cfg.norm_eps
        ops.add_rmsnorm_fwd(x=self.resid_in[l], w=pv["attn_norm"], y=self.xn1[l], rstd=self.rstd1[l], eps=eps,
                            M=M, H=H)
        self._qkv_rope(l)
        attn_ops.attention_fwd(self.qkv[l], self.attn[l], self.lse[l], B=self.B, T=T, nh=nh, nkv=nkv, d=d,
                               impl=self.attn_impl)
        self._row_parallel_add_norm(self.attn[l], wv["o_w"], x=self.resid_in[l], w=pv["ffn_norm"],
                                    out_resid=self.resid_mid[l], y=self.xn2[l], rstd=self.rstd2[l])
        self._gate_up_swiglu(l)

    def optimizer_step(self):
        if self.tp is not None and self.tp.size > 1:
            ops.seg_sqnorm(self.grad, self.cseg, self.cstart, self.cend, self.norms)
            self.tp.sum_norms_(self.norms, self.norm_w)
            ops.adamw_apply(self.master, self.grad, self.m, self.v, self.p16, self.cseg, self.cstart, self.cend,
                            self.norms, self.hp, self.loss)
            return
        ops.adamw_step(self.master, self.grad, self.m, self.v, self.p16, self.cseg, self.cstart, self.cend,
                       self.norms, self.hp, self.loss)

    def step_kernels(self):
        # gradients are zero here: cleared at allocation and by every optimizer step
        for a in range(self.A):
            self.forward_backward(a, zero_grad=False)
        self.optimizer_step()

    # ───────────────────────── CUDA graph ─────────────────────────
    def capture(self, warmup: int = 1):
        """Capture one full train step (fwd+bwd+AdamW) as a CUDA graph; replay with ``replay()``."""
        from ..utils.tracing import nvtx
        with nvtx("capture"):
            return self._capture(warmup)

    def _capture(self, warmup: int = 1):
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        # warm-up on the side stream (loads modules, sets smem attributes) without touching weights or
        # optimizer state: the step's loss is marked non-finite, so the optimizer kernels run but skip
        # the update exactly as for a NaN step (no copies of the state: large presets have no room)
        with torch.cuda.stream(s):
            for _ in range(warmup):
                for a in range(self.A):
                    self.forward_backward(a, zero_grad=False)
                self.loss[1].fill_(1.0)
                self.optimizer_step()  # skipped update; clears the gradients
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        from ..ops import _lib
        n0 = _lib.LAUNCHES[0]
        with torch.cuda.graph(g):
            self.step_kernels()
        self.kernels_per_step = _lib.LAUNCHES[0] - n0
        self.graph = g
        return g

    def step(self):
        if self.graph is not None:
            self.graph.replay()
            from ..ops import _lib
            _lib.LAUNCHES[0] += self.kernels_per_step
        else:
            self.step_kernels()

    def release_graph(self):
        self.graph = None

    # ───────────────────────── helpers ─────────────────────────
    def state_dict(self):
        return self.layout.to_state_dict(self.master)

    def flops_per_step(self) -> float:
        return self.cfg.flops_per_token(self.T) * self.M * self.A
