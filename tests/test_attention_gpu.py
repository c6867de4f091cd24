"""Flash attention kernels vs the plain fp32 PyTorch formulation (causal, GQA)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("B,T,nh,nkv,d", [(2, 64, 4, 2, 64), (2, 100, 4, 1, 64), (1, 257, 12, 4, 64),
                                          (2, 130, 16, 4, 128), (3, 64, 4, 2, 16), (1, 1023, 12, 4, 64)])
def test_attention_fwd_bwd(B, T, nh, nkv, d):
    from distrain_b200.ops import attention as A
    from distrain_b200 import ops
    torch.manual_seed(0)
    ops.clear_device_error()
    W = (nh + 2 * nkv) * d
    qkv = (torch.randn(B * T, W, device="cuda") * 1.5).bfloat16()
    out = torch.empty(B * T, nh * d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, nh, A.lse_stride(T), device="cuda")
    A.attention_fwd(qkv, out, lse, B=B, T=T, nh=nh, nkv=nkv, d=d, impl="dt")
    ref_o, ref_lse = A._torch_fwd(qkv, B, T, nh, nkv, d)
    torch.cuda.synchronize()
    assert _rel(out, ref_o) < 1e-2
    assert (lse[..., :T] - ref_lse).abs().max().item() < 1e-2
    dout = torch.randn(B * T, nh * d, device="cuda").bfloat16()
    dqkv = torch.empty_like(qkv)
    dq_acc = torch.empty(B * T, nh * d, device="cuda")
    delta = torch.empty(B, nh, A.lse_stride(T), device="cuda")
    A.attention_bwd(qkv, out, dout, lse, dqkv, dq_acc, delta, B=B, T=T, nh=nh, nkv=nkv, d=d, impl="dt")
    dq, dk, dv = A._torch_bwd(qkv, dout, B, T, nh, nkv, d)
    torch.cuda.synchronize()
    assert _rel(dqkv[:, :nh * d], dq) < 2e-2
    assert _rel(dqkv[:, nh * d:(nh + nkv) * d], dk) < 2e-2
    assert _rel(dqkv[:, (nh + nkv) * d:], dv) < 2e-2
    assert ops.device_error()[0] == 0


@pytest.mark.parametrize("B,T,nh,nkv,d", [(2, 128, 4, 2, 64), (2, 100, 4, 1, 64), (1, 1023, 12, 4, 64),
                                          (2, 300, 16, 4, 128), (1, 257, 8, 8, 128)])
def test_attention_fwd_tcgen05(B, T, nh, nkv, d):
    from distrain_b200.ops import attention as A
    from distrain_b200 import ops
    torch.manual_seed(1)
    ops.clear_device_error()
    W = (nh + 2 * nkv) * d
    qkv = (torch.randn(B * T, W, device="cuda") * 2.0).bfloat16()
    out = torch.full((B * T, nh * d), 7.0, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, nh, A.lse_stride(T), device="cuda")
    A.attention_fwd(qkv, out, lse, B=B, T=T, nh=nh, nkv=nkv, d=d, impl="tc")
    ref_o, ref_lse = A._torch_fwd(qkv, B, T, nh, nkv, d)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert _rel(out, ref_o) < 1e-2
    assert (lse[..., :T] - ref_lse).abs().max().item() < 2e-2


@pytest.mark.parametrize("B,T,nh,nkv,d", [(2, 128, 4, 2, 64), (2, 100, 4, 1, 64), (1, 1023, 12, 4, 64),
                                          (2, 300, 16, 4, 128), (1, 257, 8, 8, 128), (3, 64, 4, 2, 64)])
@pytest.mark.parametrize("impl", ["tc", "mma", "tc-ds"])
def test_attention_bwd_impls(B, T, nh, nkv, d, impl):
    from distrain_b200.ops import attention as A
    from distrain_b200 import ops
    torch.manual_seed(2)
    ops.clear_device_error()
    W = (nh + 2 * nkv) * d
    qkv = (torch.randn(B * T, W, device="cuda") * 1.5).bfloat16()
    out = torch.empty(B * T, nh * d, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(B, nh, A.lse_stride(T), device="cuda")
    A.attention_fwd(qkv, out, lse, B=B, T=T, nh=nh, nkv=nkv, d=d, impl="mma")
    dout = torch.randn(B * T, nh * d, device="cuda").bfloat16()
    dqkv = torch.full_like(qkv, 3.0)
    dq_acc = torch.empty(B * T, nh * d, device="cuda")
    delta = torch.zeros(B, nh, A.lse_stride(T), device="cuda")
    ds = None
    if impl == "tc-ds":  # dS^T stored by the key-block kernel, dQ from it
        impl = "tc"
        ds = torch.full((A.ds_bytes(B, T, nh),), 77, dtype=torch.uint8, device="cuda")
    A.attention_bwd(qkv, out, dout, lse, dqkv, dq_acc, delta, B=B, T=T, nh=nh, nkv=nkv, d=d, impl=impl, ds_buf=ds)
    dq, dk, dv = A._torch_bwd(qkv, dout, B, T, nh, nkv, d)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert _rel(dqkv[:, :nh * d], dq) < 2e-2
    assert _rel(dqkv[:, nh * d:(nh + nkv) * d], dk) < 2e-2
    assert _rel(dqkv[:, (nh + nkv) * d:], dv) < 2e-2
