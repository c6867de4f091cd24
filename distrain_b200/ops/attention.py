"""Causal GQA attention over the fused QKV activation.

``qkv`` is the [B*T, (nh+2nkv)*d] bf16 output of the QKV GEMM after bias+RoPE; query head h reads kv
head h // (nh/nkv) (reference expand_kv_heads, model.rs:127-138, done here by indexing, never by
materialising repeated K/V). ``out`` is [B*T, nh*d] bf16 (heads concatenated, the layout o_proj
consumes); ``lse`` is the fp32 log-sum-exp [B, nh, T] saved for the backward.

``impl="dt"`` runs the library's flash-attention kernels (tcgen05 forward for d = 64 / 128, mma.sync
otherwise); ``impl="mma"`` forces the mma.sync forward. ``impl="torch"`` is the plain-PyTorch
formulation used only as a test oracle on small shapes.
"""
from __future__ import annotations

import torch

import ctypes

from ._lib import lib, check, stream_ptr, ptr, register, c_int, c_void, c_float

_registered = False


def lse_stride(T: int) -> int:
    """Row stride of the [B, nh, Tp] LSE / delta buffers: T rounded up to a multiple of 4 (16-byte rows)."""
    return (T + 3) // 4 * 4


def _reg():
    global _registered
    if _registered:
        return
    register("dt_attn_fwd", [c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_int, c_float, c_void])
    register("dt_attn_bwd", [c_void, c_void, c_void, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int,
                             c_int, c_float, c_void])
    register("dt_attn_fwd_tc", [c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_int, c_float, c_void])
    register("dt_attn_bwd_delta", [c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_void])
    register("dt_attn_bwd_tc", [c_void, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_int, c_float,
                                c_void])
    register("dt_attn_bwd_tc_ds", [c_void, c_void, c_void, c_void, c_void, c_void, c_int, c_int, c_int, c_int, c_int,
                                   c_float, c_void])
    register("dt_attn_ds_bytes", [c_int, c_int, c_int], restype=ctypes.c_longlong)
    _registered = True


def bwd_kernel_for(d: int, impl: str) -> str:
    """Backward for ``impl="dt"``: tcgen05 kernels for head dims 64 / 128, mma.sync otherwise."""
    if impl == "dt":
        return "tc" if d in (64, 128) else "mma"
    return impl


def fwd_kernel_for(d: int, impl: str) -> str:
    """Which forward kernel runs for ``impl="dt"``: tcgen05 for head dims 64 / 128 (measured on B200 at
    0.18 ms vs 0.29 ms for mma.sync at B32 T1023 h12/4 d64), mma.sync otherwise. ``impl="tc"`` /
    ``"mma"`` force one."""
    if impl == "dt":
        return "tc" if d in (64, 128) else "mma"
    return impl


def attention_fwd(qkv, out, lse, *, B, T, nh, nkv, d, impl="dt", stream=None):
    scale = d ** -0.5
    if impl == "torch":
        o, l = _torch_fwd(qkv, B, T, nh, nkv, d)
        out.copy_(o)
        lse[..., :T].copy_(l)
        return
    _reg()
    kind = fwd_kernel_for(d, impl)
    if kind == "tc" and d in (64, 128):
        check(lib().dt_attn_fwd_tc(ptr(qkv), ptr(out), ptr(lse), B, T, nh, nkv, d, float(scale), stream_ptr(stream)),
              "dt_attn_fwd_tc")
        return
    check(lib().dt_attn_fwd(ptr(qkv), ptr(out), ptr(lse), B, T, nh, nkv, d, float(scale), stream_ptr(stream)),
          "dt_attn_fwd")


def ds_bytes(B: int, T: int, nh: int) -> int:
    """Size of the dS^T buffer of the tcgen05 backward: one 128 x 128 bf16 tile per causal (query block,
    key block) pair of every (batch, head)."""
    _reg()
    return int(lib().dt_attn_ds_bytes(B, T, nh))


def attention_bwd(qkv, out, dout, lse, dqkv, dq_acc, delta, *, B, T, nh, nkv, d, impl="dt", stream=None,
                  ds_buf=None):
    """dqkv <- gradients of q, k, v (same layout as qkv). ``dq_acc`` ([B*T, nh*d] fp32) and ``delta``
    ([B, nh, T] fp32) are caller-provided scratch. With ``ds_buf`` (``ds_bytes`` bytes) the tcgen05 path
    stores dS^T once in the key-block kernel and forms dQ from it with a GEMM-like kernel instead of
    recomputing S, P and dP in a second attention kernel."""
    scale = d ** -0.5
    if impl == "torch":
        dq, dk, dv = _torch_bwd(qkv, dout, B, T, nh, nkv, d)
        W = (nh + 2 * nkv) * d
        v = dqkv.view(B * T, W)
        v[:, :nh * d].copy_(dq)
        v[:, nh * d:(nh + nkv) * d].copy_(dk)
        v[:, (nh + nkv) * d:].copy_(dv)
        return
    _reg()
    if bwd_kernel_for(d, impl) == "tc" and d in (64, 128):
        sp = stream_ptr(stream)
        check(lib().dt_attn_bwd_delta(ptr(out), ptr(dout), ptr(delta), B, T, nh, d, sp), "dt_attn_bwd_delta")
        if ds_buf is not None:
            check(lib().dt_attn_bwd_tc_ds(ptr(qkv), ptr(dout), ptr(lse), ptr(delta), ptr(dqkv), ptr(ds_buf), B, T, nh,
                                          nkv, d, float(scale), sp), "dt_attn_bwd_tc_ds")
            return
        check(lib().dt_attn_bwd_tc(ptr(qkv), ptr(dout), ptr(lse), ptr(delta), ptr(dqkv), B, T, nh, nkv, d,
                                   float(scale), sp), "dt_attn_bwd_tc")
        return
    check(lib().dt_attn_bwd(ptr(qkv), ptr(out), ptr(dout), ptr(lse), ptr(dqkv), ptr(dq_acc), ptr(delta), B, T, nh,
                            nkv, d, float(scale), stream_ptr(stream)), "dt_attn_bwd")


def _split(qkv, B, T, nh, nkv, d):
    W = (nh + 2 * nkv) * d
    x = qkv.view(B, T, W).float()
    q = x[..., :nh * d].view(B, T, nh, d).transpose(1, 2)
    k = x[..., nh * d:(nh + nkv) * d].view(B, T, nkv, d).transpose(1, 2)
    v = x[..., (nh + nkv) * d:].view(B, T, nkv, d).transpose(1, 2)
    return q, k, v


def _torch_fwd(qkv, B, T, nh, nkv, d):
    q, k, v = _split(qkv, B, T, nh, nkv, d)
    g = nh // nkv
    k = k.repeat_interleave(g, dim=1)
    v = v.repeat_interleave(g, dim=1)
    s = (q @ k.transpose(-1, -2)) * d ** -0.5
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool, device=qkv.device), 1)
    s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.softmax(s, dim=-1) @ v
    return o.transpose(1, 2).reshape(B * T, nh * d).to(qkv.dtype), lse


def _torch_bwd(qkv, dout, B, T, nh, nkv, d):
    q, k, v = _split(qkv, B, T, nh, nkv, d)
    q, k, v = q.requires_grad_(), k.requires_grad_(), v.requires_grad_()
    with torch.enable_grad():
        g = nh // nkv
        kk = k.repeat_interleave(g, dim=1)
        vv = v.repeat_interleave(g, dim=1)
        s = (q @ kk.transpose(-1, -2)) * d ** -0.5
        mask = torch.triu(torch.ones(T, T, dtype=torch.bool, device=qkv.device), 1)
        s = s.masked_fill(mask, float("-inf"))
        o = torch.softmax(s, dim=-1) @ vv
        do = dout.view(B, T, nh, d).transpose(1, 2).float()
        dq, dk, dv = torch.autograd.grad(o, (q, k, v), do)
    f = lambda t, h: t.transpose(1, 2).reshape(B * T, h * d)
    return f(dq, nh), f(dk, nkv), f(dv, nkv)
