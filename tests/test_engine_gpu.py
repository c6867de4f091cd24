"""The CUDA training engine against the fp32 PyTorch oracle of the reference model."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _small_cfg(V=512, H=128, L=2, nh=4, nkv=2, F=256):
    from distrain_b200.config import ModelConfig
    return ModelConfig(hidden_dim=H, num_layers=L, num_heads=nh, num_kv_heads=nkv, ffn_hidden_dim=F, vocab_size=V,
                       max_seq_len=256, rope_theta=10000.0)


@pytest.mark.parametrize("attn_impl", ["torch", "dt"])
def test_engine_loss_and_grads_match_oracle(attn_impl):
    from distrain_b200.models.engine import TrainEngine
    from distrain_b200.models import oracle
    from distrain_b200 import ops
    if attn_impl == "dt":
        try:
            ops.lib().dt_attn_fwd
        except AttributeError:
            pytest.skip("attention kernel not built")
    torch.manual_seed(0)
    cfg = _small_cfg()
    B, S = 3, 65
    eng = TrainEngine(cfg, B, S, device="cuda", seed=1, attn_impl=attn_impl)
    tokens = torch.randint(0, cfg.vocab_size, (B, S), dtype=torch.int32)
    eng.set_tokens(tokens.cuda())
    eng.forward_backward()
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    loss = eng.loss[0].item()
    # oracle in fp32 from the bf16-rounded weights the GEMMs saw is too strict; use the fp32 master
    params = {k: v.detach().clone().double().requires_grad_() for k, v in eng.layout.views(eng.master).items()}
    ref = oracle.lm_loss(params, cfg, tokens.cuda().long(), mask_value=None)
    ref.backward()
    # the loss comes from the fp32 accumulators of the LM head (bf16 operands): within 2e-3 of the oracle
    assert abs(loss - ref.item()) < 2e-3, (loss, ref.item())
    g = eng.layout.views(eng.grad)
    for k, p in params.items():
        a, b = g[k].double(), p.grad
        rel = ((a - b).norm() / (b.norm() + 1e-12)).item()
        assert rel < 6e-2, (k, rel)


def test_engine_graph_training_decreases_loss():
    from distrain_b200.models.engine import TrainEngine
    from distrain_b200.config import OptimConfig
    torch.manual_seed(0)
    cfg = _small_cfg(V=256)
    B, S = 4, 65
    eng = TrainEngine(cfg, B, S, optim=OptimConfig(lr=3e-3), device="cuda", seed=2, attn_impl="torch")
    fixed = torch.randint(0, cfg.vocab_size, (B, S), dtype=torch.int32).cuda()
    eng.set_tokens(fixed)
    eng.capture()
    losses = []
    for _ in range(30):
        eng.step()
        losses.append(eng.loss[0].item())
    assert losses[-1] < losses[0] - 1.0, losses


def test_grad_accumulation_equals_one_large_batch():
    """2 micro-batches of B/2 accumulate to the gradients (and loss, and update) of one batch of B: same
    weights, same tokens, gradients summed in fp32 by the weight-gradient GEMMs, one AdamW step; the
    optimizer clears the gradients it has read."""
    from distrain_b200.models.engine import TrainEngine
    from distrain_b200.config import OptimConfig
    from distrain_b200 import ops
    torch.manual_seed(3)
    cfg = _small_cfg()
    B, S = 4, 65
    tokens = torch.randint(0, cfg.vocab_size, (B, S), dtype=torch.int32).cuda()
    one = TrainEngine(cfg, B, S, optim=OptimConfig(lr=1e-3), device="cuda", seed=5)
    acc = TrainEngine(cfg, B // 2, S, optim=OptimConfig(lr=1e-3), device="cuda", seed=5, grad_accum=2)
    assert torch.equal(one.master, acc.master)
    one.set_tokens(tokens)
    acc.set_tokens(tokens)
    one.forward_backward()
    acc.forward_backward(0, zero_grad=True)
    acc.forward_backward(1, zero_grad=False)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    assert abs(one.loss[0].item() - acc.loss[0].item()) < 1e-5
    ga, gb = one.layout.views(one.grad), acc.layout.views(acc.grad)
    for k in ga:
        rel = ((ga[k].double() - gb[k].double()).norm() / (ga[k].double().norm() + 1e-12)).item()
        assert rel < 1e-4, (k, rel)
    # full steps: one AdamW update each, gradients cleared afterwards. AdamW's first steps are close to
    # lr * sign(g), so gradients that differ in the last bits near zero can flip a few elements' updates:
    # compare the updates, not the weights bit for bit
    one.grad.zero_()
    acc.grad.zero_()
    m0 = one.master.clone()
    one.step_kernels()
    acc.step_kernels()
    torch.cuda.synchronize()
    assert int(one.grad.count_nonzero()) == 0 and int(acc.grad.count_nonzero()) == 0
    d1, d2 = one.master - m0, acc.master - m0
    assert ((d1 - d2).norm() / d1.norm()).item() < 2e-2
    assert abs(one.loss[0].item() - acc.loss[0].item()) < 1e-5
    # second step through the captured graph: the cleared gradients keep the two in step
    one.capture()
    acc.capture()
    m1 = one.master.clone()
    one.step()
    acc.step()
    torch.cuda.synchronize()
    assert abs(one.loss[0].item() - acc.loss[0].item()) < 1e-4
    d1, d2 = one.master - m1, acc.master - m1
    assert ((d1 - d2).norm() / d1.norm()).item() < 5e-2
