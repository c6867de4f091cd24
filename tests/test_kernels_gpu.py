"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference of the same op."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from distrain_b200 import ops
    return ops


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _no_device_error():
    ops = _ops()
    ops.clear_device_error()
    yield
    torch.cuda.synchronize()
    code, site = ops.device_error()
    assert code == 0, f"device error {code} at site {site}"


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_gemm_192_wide_tiles(a_mn, b_mn, epi):
    """192-wide output tiles (chosen for N = 768-like widths by wave quantisation) for every operand layout
    and epilogue, with partial M / K tiles."""
    ops = _ops()
    torch.manual_seed(5)
    M, N, K = 304, 576, 136  # M a multiple of 8: the row stride of an M-contiguous A
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = torch.randn(N, K, device="cuda").bfloat16()
    ref = A.float() @ B.float().t()
    a_store = A.t().contiguous() if a_mn else A
    b_store = B.t().contiguous() if b_mn else B
    if epi == 0:
        C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    else:
        C = torch.full((M, N), 0.5 if epi == 2 else 0.0, device="cuda")
    ops.gemm(a_store, b_store, C, M=M, N=N, K=K, a_mn=bool(a_mn), b_mn=bool(b_mn), epi=epi, bn=192)
    torch.cuda.synchronize()
    want = ref + 0.5 if epi == 2 else ref
    assert _rel(C, want) < (5e-3 if epi == 0 else 1e-5)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (296, 200, 136), (1000, 768, 768), (256, 1280, 768),
                                   (64, 40, 24)])
@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_gemm_bf16_out(M, N, K, a_mn, b_mn):
    ops = _ops()
    torch.manual_seed(0)
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = torch.randn(N, K, device="cuda").bfloat16()
    ref = A.float() @ B.float().t()
    a_store = A.t().contiguous() if a_mn else A
    b_store = B.t().contiguous() if b_mn else B
    C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ops.gemm(a_store, b_store, C, M=M, N=N, K=K, a_mn=bool(a_mn), b_mn=bool(b_mn))
    torch.cuda.synchronize()
    assert _rel(C, ref) < 1e-2


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("split_k", [1, 3, 0])
def test_gemm_f32_atomic_splitk(bn, split_k):
    ops = _ops()
    torch.manual_seed(1)
    M, N, K = 384, 512, 2048
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = torch.randn(N, K, device="cuda").bfloat16()
    C = torch.full((M, N), 1.0, device="cuda")
    ops.gemm(A, B, C, M=M, N=N, K=K, epi=ops.EPI_F32_ATOMIC, split_k=split_k, bn=bn, alpha=0.5)
    ref = 1.0 + 0.5 * (A.float() @ B.float().t())
    torch.cuda.synchronize()
    assert _rel(C, ref) < 1e-4


def test_gemm_f32_store_and_large():
    ops = _ops()
    torch.manual_seed(2)
    M, N, K = 4096, 4096, 1024
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = torch.randn(N, K, device="cuda").bfloat16()
    C = torch.empty(M, N, device="cuda")
    ops.gemm(A, B, C, M=M, N=N, K=K, epi=ops.EPI_F32)
    ref = A.float() @ B.float().t()
    torch.cuda.synchronize()
    assert _rel(C, ref) < 1e-4


def test_linear_helpers():
    ops = _ops()
    torch.manual_seed(3)
    M, N, K = 777, 384, 256
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda").bfloat16()
    dy = torch.randn(M, N, device="cuda").bfloat16()
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    dx = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
    dw = torch.zeros(N, K, device="cuda")
    ops.linear_fwd(x, w, y)
    ops.linear_dgrad(dy, w, dx)
    ops.linear_wgrad(dy, x, dw)
    torch.cuda.synchronize()
    assert _rel(y, x.float() @ w.float().t()) < 1e-2
    assert _rel(dx, dy.float() @ w.float()) < 1e-2
    assert _rel(dw, dy.float().t() @ x.float()) < 1e-3


@pytest.mark.parametrize("H", [64, 768, 2048, 5120])
def test_add_rmsnorm_fwd_bwd(H):
    ops = _ops()
    torch.manual_seed(4)
    M, eps = 97, 1e-5
    x = torch.randn(M, H, device="cuda")
    br = torch.randn(M, H, device="cuda").bfloat16()
    w = torch.rand(H, device="cuda") + 0.5
    scale = torch.tensor([1.7], device="cuda")
    out_resid = torch.empty(M, H, device="cuda")
    y = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    rstd = torch.empty(M, device="cuda")
    ops.add_rmsnorm_fwd(x=x, br=br, w=w, scale=scale, out_resid=out_resid, y=y, rstd=rstd, eps=eps, M=M, H=H)
    r = x + br.float()
    ref_y = r * torch.rsqrt(r.pow(2).mean(-1, keepdim=True) + eps) * w * scale
    torch.cuda.synchronize()
    assert torch.allclose(out_resid, r)
    assert _rel(y, ref_y) < 8e-3
    # backward vs autograd
    rr = r.clone().requires_grad_()
    ww = w.clone().requires_grad_()
    ss = scale.clone().requires_grad_()
    out = rr * torch.rsqrt(rr.pow(2).mean(-1, keepdim=True) + eps) * ww * ss
    dy = torch.randn(M, H, device="cuda").bfloat16()
    out.backward(dy.float())
    prev = torch.randn(M, H, device="cuda")
    dres = prev.clone()
    d16 = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    dw = torch.zeros(H, device="cuda")
    ds = torch.zeros(1, device="cuda")
    ops.rmsnorm_bwd(dy=dy, x=r, rstd=rstd, w=w, scale=scale, dresid_in=dres, dresid_out=dres, dresid16=d16, dw=dw,
                    dscale=ds, M=M, H=H)
    torch.cuda.synchronize()
    assert _rel(dres, prev + rr.grad) < 1e-4
    assert _rel(d16, prev + rr.grad) < 8e-3
    assert _rel(dw, ww.grad) < 1e-4
    assert _rel(ds, ss.grad) < 1e-4


def test_embedding_gather_and_bwd():
    ops = _ops()
    torch.manual_seed(5)
    B, S, V, H = 3, 17, 50, 64
    T = S - 1
    M = B * T
    ids = torch.randint(0, V, (B, S), device="cuda", dtype=torch.int32)
    E = torch.randn(V, H, device="cuda")
    w = torch.ones(H, device="cuda")
    resid = torch.empty(M, H, device="cuda")
    y = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    rstd = torch.empty(M, device="cuda")
    ops.add_rmsnorm_fwd(emb=E, ids=ids, T=T, S=S, w=w, out_resid=resid, y=y, rstd=rstd, eps=1e-5, M=M, H=H)
    ref = E[ids[:, :-1].long()].reshape(M, H)
    g = torch.randn(M, H, device="cuda")
    dE = torch.zeros(V, H, device="cuda")
    ops.embedding_bwd(g, ids, dE, T=T, S=S, M=M, H=H)
    ref_dE = torch.zeros(V, H, device="cuda").index_add_(0, ids[:, :-1].reshape(-1).long(), g)
    torch.cuda.synchronize()
    assert torch.allclose(resid, ref)
    assert torch.allclose(dE, ref_dE, atol=1e-5)


@pytest.mark.parametrize("nh,nkv,d", [(4, 2, 16), (12, 4, 64), (16, 4, 128)])
def test_rope_fwd_bwd(nh, nkv, d):
    from distrain_b200.models.oracle import apply_rope, rope_tables
    from distrain_b200.config import ModelConfig
    ops = _ops()
    torch.manual_seed(6)
    B, T = 2, 33
    M, W = B * T, (nh + 2 * nkv) * d
    cfg = ModelConfig(hidden_dim=nh * d, num_heads=nh, num_kv_heads=nkv, rope_theta=10000.0)
    cos, sin = rope_tables(cfg, T)
    cos, sin = cos.cuda(), sin.cuda()
    qkv = torch.randn(M, W, device="cuda").bfloat16()
    bias = torch.randn(W, device="cuda") * 0.1
    x = (qkv.float() + bias).view(B, T, nh + 2 * nkv, d)
    ref = torch.cat([apply_rope(x[:, :, :nh + nkv], cos, sin), x[:, :, nh + nkv:]], dim=2).reshape(M, W)
    out = qkv.clone()
    ops.rope_fwd(out, bias, cos, sin, M=M, T=T, nh=nh, nkv=nkv, d=d)
    torch.cuda.synchronize()
    assert _rel(out, ref) < 8e-3
    # backward: gradient of sum(g * rope(x + b))
    xx = (qkv.float()).view(B, T, nh + 2 * nkv, d).requires_grad_()
    bb = bias.clone().requires_grad_()
    y = xx + bb.view(nh + 2 * nkv, d)
    y = torch.cat([apply_rope(y[:, :, :nh + nkv], cos, sin), y[:, :, nh + nkv:]], dim=2).reshape(M, W)
    g = torch.randn(M, W, device="cuda").bfloat16()
    y.backward(g.float())
    # bias gradient by atomics and by per-block scratch rows + one reduction; both add into dbias
    for part in (None, torch.full((ops.rope_bwd_scratch(M, nh, nkv, d),), float("nan"), device="cuda")):
        dq = g.clone()
        db = torch.full((W,), 0.5, device="cuda")
        ops.rope_bwd(dq, db, cos, sin, M=M, T=T, nh=nh, nkv=nkv, d=d, part=part)
        torch.cuda.synchronize()
        assert _rel(dq, xx.grad.reshape(M, W)) < 8e-3
        assert _rel(db - 0.5, bb.grad) < 1e-4


def test_swiglu_fwd_bwd():
    ops = _ops()
    torch.manual_seed(7)
    M, F = 129, 256
    gu = torch.randn(M, 2 * F, device="cuda").bfloat16()
    h = torch.empty(M, F, device="cuda", dtype=torch.bfloat16)
    ops.swiglu_fwd(gu, h, M=M, F=F)
    g, u = gu.float()[:, :F].requires_grad_(), gu.float()[:, F:].requires_grad_()
    ref = torch.nn.functional.silu(g) * u
    dh = torch.randn(M, F, device="cuda").bfloat16()
    ref.backward(dh.float())
    dgu = torch.empty_like(gu)
    ops.swiglu_bwd(dh, gu, dgu, M=M, F=F)
    torch.cuda.synchronize()
    assert _rel(h, ref) < 8e-3
    assert _rel(dgu[:, :F], g.grad) < 1e-2
    assert _rel(dgu[:, F:], u.grad) < 1e-2


@pytest.mark.parametrize("B,T,nh,nkv,d,K,bias", [(3, 65, 4, 2, 64, 160, True), (2, 1023, 12, 4, 64, 768, True),
                                                  (2, 100, 4, 2, 128, 256, False), (1, 300, 2, 1, 128, 64, True)])
def test_gemm_qkv_rope_fused(B, T, nh, nkv, d, K, bias):
    """QKV GEMM with bias + rotate-half RoPE in its epilogue vs fp32 torch (GEMM, bias, rotation by
    position row % T with the engine's fp32 tables)."""
    from distrain_b200.config import ModelConfig
    from distrain_b200.models.oracle import rope_tables
    ops = _ops()
    torch.manual_seed(13)
    M, W = B * T, (nh + 2 * nkv) * d
    cfg = ModelConfig(hidden_dim=nh * d, num_layers=1, num_heads=nh, num_kv_heads=nkv, ffn_hidden_dim=64,
                      vocab_size=64, max_seq_len=T, rope_theta=10000.0)
    cos, sin = rope_tables(cfg, T)
    cos, sin = cos.cuda().contiguous(), sin.cuda().contiguous()
    x = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    w = (torch.randn(W, K, device="cuda") / K ** 0.5).bfloat16()
    b = torch.randn(W, device="cuda") * 0.1 if bias else None
    out = torch.full((M, W), 7.0, device="cuda", dtype=torch.bfloat16)
    ops.gemm_qkv_rope(x, w, b, cos, sin, out, T=T, d=d, rot_cols=(nh + nkv) * d)
    torch.cuda.synchronize()
    z = x.float() @ w.float().t() + (b if bias else 0.0)
    t = torch.arange(M, device="cuda") % T
    c, s_ = cos[t], sin[t]  # [M, d/2]
    ref = z.clone()
    half = d // 2
    for h in range(nh + nkv):
        a, q = z[:, h * d:h * d + half], z[:, h * d + half:(h + 1) * d]
        ref[:, h * d:h * d + half] = a * c - q * s_
        ref[:, h * d + half:(h + 1) * d] = a * s_ + q * c
    assert _rel(out, ref) < 5e-3
    assert _rel(out[:, (nh + nkv) * d:], ref[:, (nh + nkv) * d:]) < 5e-3


@pytest.mark.parametrize("M,F,K", [(129, 192, 160), (300, 256, 768), (1000, 2048, 768), (64, 64, 64)])
def test_gemm_swiglu_fwd_fused(M, F, K):
    """gate|up GEMM with the SwiGLU activation in its epilogue vs fp32 torch (partial row, column and
    K tiles included)."""
    ops = _ops()
    torch.manual_seed(11)
    x = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    w = (torch.randn(2 * F, K, device="cuda") / K ** 0.5).bfloat16()
    gu = torch.full((M, 2 * F), 7.0, device="cuda", dtype=torch.bfloat16)
    h = torch.full((M, F), 7.0, device="cuda", dtype=torch.bfloat16)
    ops.gemm_swiglu_fwd(x, w, gu, h)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    g, u = ref[:, :F], ref[:, F:]
    assert _rel(gu, ref) < 5e-3
    assert _rel(h, torch.nn.functional.silu(g) * u) < 8e-3


@pytest.mark.parametrize("M,F,K", [(129, 192, 160), (300, 256, 768), (1000, 2048, 768), (64, 64, 64)])
def test_gemm_swiglu_bwd_fused(M, F, K):
    """down-projection data gradient with the SwiGLU backward in its epilogue (dh never stored) vs fp32
    torch autograd through silu(g) * u."""
    ops = _ops()
    torch.manual_seed(12)
    dy = torch.randn(M, K, device="cuda").bfloat16()
    wd = (torch.randn(K, F, device="cuda") / K ** 0.5).bfloat16()
    gu = torch.randn(M, 2 * F, device="cuda").bfloat16()
    dgu = torch.full((M, 2 * F), 7.0, device="cuda", dtype=torch.bfloat16)
    ops.gemm_swiglu_bwd(dy, wd, gu, dgu)
    torch.cuda.synchronize()
    dh = dy.float() @ wd.float()
    g, u = gu.float()[:, :F].requires_grad_(), gu.float()[:, F:].requires_grad_()
    (torch.nn.functional.silu(g) * u).backward(dh)
    assert _rel(dgu[:, :F], g.grad) < 1e-2
    assert _rel(dgu[:, F:], u.grad) < 1e-2


@pytest.mark.parametrize("rows,V,K,T", [(300, 512, 128, 64), (1023, 32768, 768, 1023), (200, 1000, 64, 50)])
def test_logits_lse_and_cross_entropy(rows, V, K, T):
    """LM-head GEMM with fp32 softmax statistics in its epilogue + the cross-entropy pass that uses them:
    the loss per row equals the fp32 log-sum-exp minus the fp32 target logit of the same product (no bf16
    rounding of the logits enters the loss), the logits are replaced by the scaled softmax - onehot."""
    ops = _ops()
    torch.manual_seed(21)
    S = T + 1
    nb = (rows + T - 1) // T
    ids = torch.randint(0, V, (nb, S), device="cuda", dtype=torch.int32)
    x = (torch.randn(rows, K, device="cuda") * 0.5).bfloat16()
    e = (torch.randn(V, K, device="cuda") / K ** 0.5 * 3).bfloat16()
    logits = torch.empty(rows, V, device="cuda", dtype=torch.bfloat16)
    part = torch.empty(2 * ops.lse_parts(rows, V), device="cuda")
    tl = torch.empty(rows, device="cuda")
    loss = torch.empty(rows, device="cuda")
    r0 = 0
    ops.gemm_logits_lse(x, e, logits, part, tl, ids, rows=rows, V=V, K=K, T=T, S=S, r0=r0)
    ref = x.float() @ e.float().t()
    torch.cuda.synchronize()
    assert _rel(logits, ref) < 5e-3
    g = torch.arange(rows, device="cuda") + r0
    tgt = ids[g // T, g % T + 1].long()
    ref_tl = ref.gather(1, tgt[:, None])[:, 0]
    assert torch.allclose(tl, ref_tl, rtol=1e-4, atol=1e-4)
    ops.ce_lse_bwd(logits, part, tl, ids, loss, rows=rows, V=V, T=T, S=S, r0=r0, grad_scale=0.5)
    torch.cuda.synchronize()
    ref_loss = torch.logsumexp(ref, dim=1) - ref_tl
    assert (loss - ref_loss).abs().max().item() < 1e-4
    p = torch.softmax(ref, dim=1)
    p[torch.arange(rows), tgt] -= 1.0
    assert _rel(logits, 0.5 * p) < 2e-2


@pytest.mark.parametrize("V", [32768, 512, 256])
def test_cross_entropy(V):
    ops = _ops()
    torch.manual_seed(8)
    B, S = 2, 9
    T = S - 1
    M = B * T
    ids = torch.randint(0, V, (B, S), device="cuda", dtype=torch.int32)
    z = (torch.randn(M, V, device="cuda") * 3).bfloat16()
    zz = z.float().requires_grad_()
    tgt = ids[:, 1:].reshape(-1).long()
    loss = torch.nn.functional.cross_entropy(zz, tgt)
    loss.backward()
    rows = torch.empty(M, device="cuda")
    zg = z.clone()
    ops.ce_fwd_bwd(zg, ids, rows, T=T, S=S, r0=0, rows=M, V=V, grad_scale=1.0 / M)
    out = torch.zeros(4, device="cuda")
    ops.loss_reduce(rows, M, 1.0 / M, out)
    torch.cuda.synchronize()
    assert abs(out[0].item() - loss.item()) < 1e-3 * max(1.0, loss.item())
    assert out[1].item() == 0.0
    assert _rel(zg, zz.grad) < 1e-2


def test_adamw_matches_reference():
    from distrain_b200.config import ModelConfig
    from distrain_b200.models.params import ParamLayout, init_flat
    from distrain_b200.models.oracle import AdamWRef
    ops = _ops()
    cfg = ModelConfig(hidden_dim=64, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=128, vocab_size=256)
    L = ParamLayout(cfg)
    flat = init_flat(L, 0.02, 0).cuda()
    grads = torch.randn(L.total, device="cuda") * 0.5
    mask = torch.zeros(L.total, dtype=torch.bool, device="cuda")
    for e in L.entries:
        mask[e.offset:e.offset + e.numel] = True
    grads = grads * mask
    p = flat.clone()
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    p16 = torch.empty(L.total, dtype=torch.bfloat16, device="cuda")
    cseg, cstart, cend, nseg = L.chunk_tables("cuda")
    norms = torch.zeros(nseg, device="cuda")
    hp = torch.zeros(16, device="cuda")
    hp[0], hp[1], hp[2], hp[3], hp[4], hp[7] = 1e-3, 0.9, 0.999, 1e-5, 0.1, 1.0
    loss = torch.zeros(4, device="cuda")
    ref_params = {k: t.clone() for k, t in L.views(flat.clone()).items()}
    opt = AdamWRef(ref_params, lr=1e-3, clip=1.0)
    for it in range(3):
        ops.adamw_step(p, grads, m, v, p16, cseg, cstart, cend, norms, hp, loss)
        for k, t in ref_params.items():
            t.grad = L.view(grads, k).clone()
        opt.step()
    torch.cuda.synchronize()
    got = L.views(p)
    for k, t in ref_params.items():
        assert torch.allclose(got[k], t, atol=1e-6, rtol=1e-5), k
    assert torch.equal(p16[mask].float(), p[mask].bfloat16().float())
    # NaN loss flag skips the update
    before = p.clone()
    loss[1] = 1.0
    ops.adamw_step(p, grads, m, v, p16, cseg, cstart, cend, norms, hp, loss)
    torch.cuda.synchronize()
    assert torch.equal(before, p)


_PAIR_SCRIPT = r"""
import sys, torch
from distrain_b200 import ops
torch.manual_seed(7)
out = {}
for (M, N, K, a_mn, b_mn, epi) in [(300, 512, 768, 0, 0, 0), (1000, 768, 136, 1, 1, 1), (257, 1280, 512, 0, 1, 2)]:
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = torch.randn(N, K, device="cuda").bfloat16()
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    C = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16 if epi == 0 else torch.float32)
    ops.gemm(a, b, C, M=M, N=N, K=K, a_mn=bool(a_mn), b_mn=bool(b_mn), epi=epi, bn=256)
    out[(M, N, K)] = C.float().cpu()
torch.cuda.synchronize()
assert ops.device_error()[0] == 0
torch.save(out, sys.argv[1])
"""


@pytest.mark.parametrize("mode", ["0", "2"])
def test_gemm_256_wide_single_cta_and_pair_paths(tmp_path, mode):
    """256-wide tiles run on CTA pairs by default (DT_GEMM_PAIR unset / 2); DT_GEMM_PAIR=0 keeps them on
    single CTAs. Both paths (in child processes, the mode is read once) against the fp32 product."""
    import os
    import subprocess
    import sys
    path = str(tmp_path / f"out{mode}.pt")
    env = dict(os.environ, DT_GEMM_PAIR=mode)
    r = subprocess.run([sys.executable, "-c", _PAIR_SCRIPT, path], env=env, capture_output=True, text=True,
                       timeout=300, cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0, r.stderr[-2000:]
    out = torch.load(path)
    torch.manual_seed(7)
    for (M, N, K, a_mn, b_mn, epi) in [(300, 512, 768, 0, 0, 0), (1000, 768, 136, 1, 1, 1), (257, 1280, 512, 0, 1, 2)]:
        A = torch.randn(M, K, device="cuda").bfloat16()
        B = torch.randn(N, K, device="cuda").bfloat16()
        ref = (A.float() @ B.float().t()).cpu()
        assert _rel(out[(M, N, K)], ref) < (1e-2 if epi == 0 else 1e-4), (M, N, K, mode)
