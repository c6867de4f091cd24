"""Python entry points of the sm_100a kernel library.

Each function takes torch tensors that already live on the GPU, launches the matching C-ABI
launcher on the current stream and raises ``KernelError`` on any launch/argument failure.
No function here allocates except where documented (``attention`` scratch is caller-provided).
"""
from __future__ import annotations

import torch

from ._lib import lib, check, stream_ptr, ptr, device_error, clear_device_error, KernelError  # noqa: F401

EPI_BF16, EPI_F32, EPI_F32_ATOMIC = 0, 1, 2


def gemm(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, *, M: int, N: int, K: int, a_mn: bool = False,
         b_mn: bool = False, lda: int = None, ldb: int = None, ldc: int = None, epi: int = None,
         alpha: float = 1.0, split_k: int = 0, bn: int = 0, stream=None):
    """C[M,N] (op)= alpha * A[M,K] . B[N,K]^T on tcgen05 tensor cores.

    ``a_mn`` False: A(m,k) = a[m*lda + k]; True: A(m,k) = a[k*lda + m]. Same for B with n.
    ``epi``: EPI_BF16 (store bf16), EPI_F32 (store fp32), EPI_F32_ATOMIC (C += result, fp32; split-K allowed).
    """
    assert a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16
    if epi is None:
        epi = EPI_BF16 if c.dtype == torch.bfloat16 else EPI_F32
    if lda is None:
        lda = M if a_mn else K
    if ldb is None:
        ldb = N if b_mn else K
    if ldc is None:
        ldc = N
    rc = lib().dt_gemm_bf16(a.data_ptr(), int(a_mn), lda, b.data_ptr(), int(b_mn), ldb, c.data_ptr(), ldc, M, N, K,
                            epi, float(alpha), int(split_k), int(bn), stream_ptr(stream))
    check(rc, "dt_gemm_bf16")


def linear_fwd(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, stream=None):
    """out[M,N] = x[M,K] @ w[N,K]^T (bf16 in/out)."""
    M, K = x.shape
    N = w.shape[0]
    gemm(x, w, out, M=M, N=N, K=K, stream=stream)


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, dx: torch.Tensor, stream=None):
    """dx[M,K] = dy[M,N] @ w[N,K]."""
    M, N = dy.shape
    K = w.shape[1]
    gemm(dy, w, dx, M=M, N=K, K=N, b_mn=True, ldb=K, stream=stream)


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, dw: torch.Tensor, alpha: float = 1.0, stream=None):
    """dw[N,K] += alpha * dy[M,N]^T @ x[M,K]   (fp32 accumulate, split-K as needed)."""
    M, N = dy.shape
    K = x.shape[1]
    gemm(dy, x, dw, M=N, N=K, K=M, a_mn=True, lda=N, b_mn=True, ldb=K, ldc=K, epi=EPI_F32_ATOMIC, alpha=alpha,
         stream=stream)


def linear_peer(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor, peer_out: int, peer_arrivals: int,
                done_ctas: int, *, dgrad: bool = False, stream=None):
    """Row-parallel forward (``dgrad`` False: out = a @ w^T) or column-parallel data gradient (``dgrad`` True:
    out = a @ w) whose every output box is also stored into the tensor-parallel peer's receive buffer
    ``peer_out`` (a device address on the peer GPU), then signalled on ``peer_arrivals``."""
    M = a.shape[0]
    if dgrad:
        N, K, b_mn, ldb = w.shape[1], w.shape[0], 1, w.shape[1]
    else:
        N, K, b_mn, ldb = w.shape[0], w.shape[1], 0, w.shape[1]
    check(lib().dt_gemm_bf16_peer(ptr(a), 0, K, ptr(w), b_mn, ldb, ptr(out), N, M, N, K, 1.0, 0, peer_out,
                                  peer_arrivals, done_ctas, stream_ptr(stream)), "dt_gemm_bf16_peer")


def add_rmsnorm_fwd_tp(*, x, br, br2, w, y, rstd, eps, M, H, arrivals, consumed, done_blocks, scale=None,
                       out_resid=None, stream=None):
    """resid_out = x + br + br2 (br2: the peer's partial, waited for on the counters); y = rmsnorm(...)."""
    check(lib().dt_add_rmsnorm_fwd_tp(ptr(x), ptr(br), ptr(br2), ptr(w), ptr(scale), ptr(out_resid), ptr(y),
                                      ptr(rstd), M, H, float(eps), arrivals, consumed, done_blocks,
                                      stream_ptr(stream)), "dt_add_rmsnorm_fwd_tp")


def rmsnorm_bwd_tp(*, dy, dy2, x, rstd, w, dresid_out, dw, M, H, arrivals, consumed, done_blocks, scale=None,
                   dresid_in=None, dresid16=None, dscale=None, stream=None):
    check(lib().dt_rmsnorm_bwd_tp(ptr(dy), ptr(dy2), ptr(x), ptr(rstd), ptr(w), ptr(scale), ptr(dresid_in),
                                  ptr(dresid_out), ptr(dresid16), ptr(dw), ptr(dscale), M, H, arrivals, consumed,
                                  done_blocks, stream_ptr(stream)), "dt_rmsnorm_bwd_tp")


def add_rmsnorm_fwd(*, y, rstd, w, eps, M, H, x=None, br=None, emb=None, ids=None, T=1, S=1, scale=None,
                    out_resid=None, stream=None):
    check(lib().dt_add_rmsnorm_fwd(ptr(x), ptr(br), ptr(emb), ptr(ids), T, S, ptr(w), ptr(scale), ptr(out_resid),
                                   ptr(y), ptr(rstd), M, H, float(eps), stream_ptr(stream)), "dt_add_rmsnorm_fwd")


def rmsnorm_bwd(*, dy, x, rstd, w, dresid_out, dw, M, H, scale=None, dresid_in=None, dresid16=None, dscale=None,
                stream=None):
    check(lib().dt_rmsnorm_bwd(ptr(dy), ptr(x), ptr(rstd), ptr(w), ptr(scale), ptr(dresid_in), ptr(dresid_out),
                               ptr(dresid16), ptr(dw), ptr(dscale), M, H, stream_ptr(stream)), "dt_rmsnorm_bwd")


def embedding_bwd(g, ids, dE, *, T, S, M, H, stream=None):
    check(lib().dt_embedding_bwd(ptr(g), ptr(ids), T, S, ptr(dE), M, H, stream_ptr(stream)), "dt_embedding_bwd")


def rope_fwd(qkv, bias, cos, sin, *, M, T, nh, nkv, d, stream=None):
    check(lib().dt_rope_fwd(ptr(qkv), ptr(bias), ptr(cos), ptr(sin), M, T, nh, nkv, d, stream_ptr(stream)),
          "dt_rope_fwd")


def rope_bwd_scratch(M, nh, nkv, d) -> int:
    """fp32 elements of the ``part`` scratch of ``rope_bwd`` for M rows."""
    from ._lib import register
    import ctypes
    f = register("dt_rope_bwd_scratch", [ctypes.c_int] * 4, restype=ctypes.c_longlong)
    return int(f(M, nh, nkv, d))


def rope_bwd(dqkv, dbias, cos, sin, *, M, T, nh, nkv, d, part=None, stream=None):
    """Inverse rotation of the QKV gradient in place; dbias += its column sums. With ``part``
    (``rope_bwd_scratch`` fp32 elements) the sums go through per-block scratch rows and one reduction
    kernel instead of atomics on the same addresses from every block."""
    check(lib().dt_rope_bwd(ptr(dqkv), ptr(dbias), ptr(part), ptr(cos), ptr(sin), M, T, nh, nkv, d,
                            stream_ptr(stream)), "dt_rope_bwd")
    if part is not None and dbias is not None:
        from . import _lib
        _lib.LAUNCHES[0] += 1  # the column-sum reduction


def gemm_qkv_rope(x, w, bias, cos, sin, out, *, T, d, rot_cols, stream=None):
    """out[M, N] = rope(x[M, K] @ w[N, K]^T + bias) in one tcgen05 GEMM: the epilogue adds the bias and
    rotates every head whose columns lie below ``rot_cols`` (q and k heads) by the position row % T
    (fp32 cos / sin tables [T, d/2]); d = 64 or 128."""
    M, K = x.shape
    N = w.shape[0]
    check(lib().dt_gemm_qkv_rope(ptr(x), K, ptr(w), K, ptr(bias), ptr(cos), ptr(sin), ptr(out), M, N, K, T, d,
                                 rot_cols, 0, stream_ptr(stream)), "dt_gemm_qkv_rope")


def gemm_swiglu_fwd(x, w_gu, gu, h, stream=None):
    """gu[M, 2F] = x[M, K] @ w_gu[2F, K]^T (gate | up, bf16) and h[M, F] = silu(gate) * up in the same
    tcgen05 GEMM (its epilogue), from the fp32 accumulators. F a multiple of 64."""
    M, K = x.shape
    F = h.shape[1]
    assert w_gu.shape == (2 * F, K) and gu.shape == (M, 2 * F) and h.shape == (M, F)
    check(lib().dt_gemm_swiglu_fwd(ptr(x), K, ptr(w_gu), K, ptr(gu), ptr(h), M, F, K, stream_ptr(stream)),
          "dt_gemm_swiglu_fwd")


def gemm_swiglu_bwd(dy, w_down, gu, dgu, stream=None):
    """dgu[M, 2F] = SwiGLU backward of dh = dy[M, K] @ w_down[K, F] against the saved gu (dh itself is
    never stored): dgate = dh * up * silu'(gate), dup = dh * silu(gate). F a multiple of 64."""
    M, K = dy.shape
    F = w_down.shape[1]
    assert w_down.shape == (K, F) and gu.shape == (M, 2 * F) and dgu.shape == (M, 2 * F)
    check(lib().dt_gemm_swiglu_bwd(ptr(dy), K, ptr(w_down), F, ptr(gu), ptr(dgu), M, F, K, 0, stream_ptr(stream)),
          "dt_gemm_swiglu_bwd")


def swiglu_fwd(gu, h, *, M, F, stream=None):
    check(lib().dt_swiglu_fwd(ptr(gu), ptr(h), M, F, stream_ptr(stream)), "dt_swiglu_fwd")


def swiglu_bwd(dh, gu, dgu, *, M, F, stream=None):
    check(lib().dt_swiglu_bwd(ptr(dh), ptr(gu), ptr(dgu), M, F, stream_ptr(stream)), "dt_swiglu_bwd")


def ce_fwd_bwd(logits, ids, loss_rows, *, T, S, r0, rows, V, ld=None, grad_scale=1.0, stream=None):
    check(lib().dt_ce_fwd_bwd(ptr(logits), V if ld is None else ld, ptr(ids), T, S, r0, rows, ptr(loss_rows), V,
                              float(grad_scale), stream_ptr(stream)), "dt_ce_fwd_bwd")


def lse_parts(rows: int, V: int) -> int:
    """float2 entries of the softmax-statistics buffer ``gemm_logits_lse`` fills for ``rows`` rows."""
    return 2 * ((V + 255) // 256) * rows


def gemm_logits_lse(x, emb, logits, part, tgt_logit, ids, *, rows, V, K, T, S, r0, stream=None):
    """logits[rows, V] = x[rows, K] @ emb[V, K]^T (bf16) and, from the fp32 accumulators, the per-row
    softmax statistics (``part``: fp32 pairs, ``lse_parts(rows, V)`` of them) and the fp32 logit of each
    row's target token (``tgt_logit``); target of global row r0 + r = ids[b*S + t + 1]."""
    check(lib().dt_gemm_logits_lse(ptr(x), x.stride(0), ptr(emb), emb.stride(0), ptr(logits), logits.stride(0), rows,
                                   V, K, ptr(part), ptr(tgt_logit), ptr(ids), T, S, r0, stream_ptr(stream)),
          "dt_gemm_logits_lse")


def ce_lse_bwd(logits, part, tgt_logit, ids, loss_rows, *, rows, V, T, S, r0, grad_scale, row_w=None, stream=None):
    """Cross-entropy of ``rows`` rows from ``gemm_logits_lse``'s statistics: loss_rows = lse - target logit
    (fp32) and the logits replaced in place by grad_scale * (softmax - onehot), times ``row_w[r0 + r]``
    when per-row weights are given (fp32, indexed like the rows of ``ids``)."""
    np_ = lse_parts(1, V)
    check(lib().dt_ce_lse_bwd(ptr(logits), logits.stride(0), ptr(part), np_, rows, ptr(tgt_logit), ptr(ids), T, S, r0,
                              ptr(loss_rows), V, float(grad_scale), ptr(row_w), stream_ptr(stream)), "dt_ce_lse_bwd")


def loss_reduce(loss_rows, n, scale, out, w=None, stream=None):
    """out[0] = scale * sum(loss_rows[:n]) (weighted by ``w[:n]`` when given; zero-weight rows are dropped)."""
    check(lib().dt_loss_reduce(ptr(loss_rows), n, float(scale), ptr(out), ptr(w), stream_ptr(stream)),
          "dt_loss_reduce")


def adamw_step(p, g, m, v, p16, cseg, cstart, cend, norms, hp, loss_flag=None, stream=None):
    check(lib().dt_adamw_step(ptr(p), ptr(g), ptr(m), ptr(v), ptr(p16), ptr(cseg), ptr(cstart), ptr(cend),
                              cseg.numel(), ptr(norms), norms.numel(), ptr(hp), ptr(loss_flag), stream_ptr(stream)),
          "dt_adamw_step")


def adamw_apply(p, g, m, v, p16, cseg, cstart, cend, norms, hp, loss_flag=None, stream=None):
    """AdamW prepare + update with precomputed per-segment squared norms (tensor-parallel clipping)."""
    check(lib().dt_adamw_apply(ptr(p), ptr(g), ptr(m), ptr(v), ptr(p16), ptr(cseg), ptr(cstart), ptr(cend),
                               cseg.numel(), ptr(norms), norms.numel(), ptr(hp), ptr(loss_flag), stream_ptr(stream)),
          "dt_adamw_apply")


def seg_sqnorm(g, cseg, cstart, cend, norms, stream=None):
    check(lib().dt_seg_sqnorm(ptr(g), ptr(cseg), ptr(cstart), ptr(cend), cseg.numel(), ptr(norms), norms.numel(),
                              stream_ptr(stream)), "dt_seg_sqnorm")


def cast_bf16(x, y, stream=None):
    check(lib().dt_cast_bf16(ptr(x), ptr(y), x.numel(), stream_ptr(stream)), "dt_cast_bf16")
