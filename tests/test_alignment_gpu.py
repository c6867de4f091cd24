"""Post-training on the CUDA engine: per-row loss weights against the fp64 oracle, the forward-only loss
pass, and short SFT / DPO runs on synthetic data."""
import json
import math
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _small_cfg(V=512):
    from distrain_b200.config import ModelConfig
    return ModelConfig(hidden_dim=128, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=256, vocab_size=V,
                       max_seq_len=256, rope_theta=10000.0)


def _row_ce(p, cfg, ids):
    from distrain_b200.models import oracle
    ids = ids.long()
    z = oracle.logits_fn(p, cfg, ids[:, :-1], mask_value=None)
    return -torch.log_softmax(z, dim=-1).gather(-1, ids[:, 1:, None])[..., 0]


@pytest.mark.parametrize("A,signed", [(1, False), (2, False), (1, True), (2, True)])
def test_weighted_loss_and_grads_match_oracle(A, signed):
    """Per-row weights (zeros included; positive, or of both signs) over A micro-batches: the step's loss
    is sum w * ce and the gradients are those of that sum. With signed weights the scalar output-scale
    gradient is a sum that mostly cancels, so the bf16 forward's error dominates its relative error: the
    scalar is left out of that case."""
    from distrain_b200.models.engine import TrainEngine
    from distrain_b200 import ops
    torch.manual_seed(4)
    cfg = _small_cfg()
    B, S = 2, 65
    eng = TrainEngine(cfg, B, S, device="cuda", seed=7, grad_accum=A, loss_weights=True)
    tokens = torch.randint(0, cfg.vocab_size, (A * B, S), dtype=torch.int32).cuda()
    w = (torch.randn(A * B, S - 1) if signed else torch.rand(A * B, S - 1) + 0.5) / (A * B * (S - 1))
    w[:, :10] = 0.0
    eng.set_tokens(tokens)
    eng.set_loss_weights(w.cuda())
    for a in range(A):
        eng.forward_backward(a, zero_grad=a == 0)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    params = {k: v.detach().clone().double().requires_grad_() for k, v in eng.layout.views(eng.master).items()}
    ref = (w.cuda().double() * _row_ce(params, cfg, tokens)).sum()
    ref.backward()
    assert abs(eng.loss[0].item() - ref.item()) < 2e-3 * float(w.abs().sum()), (eng.loss[0].item(), ref.item())
    g = eng.layout.views(eng.grad)
    for k, p in params.items():
        if signed and p.numel() == 1:
            continue
        rel = ((g[k].double() - p.grad).norm() / (p.grad.norm() + 1e-12)).item()
        assert rel < 6e-2, (k, rel)


def test_forward_loss_rows_match_oracle_and_leave_state():
    from distrain_b200.models.engine import TrainEngine
    from distrain_b200 import ops
    torch.manual_seed(5)
    cfg = _small_cfg()
    B, S, A = 3, 65, 2
    eng = TrainEngine(cfg, B, S, device="cuda", seed=8, grad_accum=A, loss_weights=True)
    tokens = torch.randint(0, cfg.vocab_size, (A * B, S), dtype=torch.int32).cuda()
    eng.set_tokens(tokens)
    m0, loss0 = eng.master.clone(), eng.loss.clone()
    rows = torch.cat([eng.forward_loss(a).clone() for a in range(A)]).view(A * B, S - 1)
    torch.cuda.synchronize()
    assert ops.device_error()[0] == 0
    params = {k: v.detach().clone().double() for k, v in eng.layout.views(eng.master).items()}
    with torch.no_grad():
        ref = _row_ce(params, cfg, tokens)
    err = (rows.double() - ref).abs()
    assert err.max().item() < 5e-2 and err.mean().item() < 5e-3, (err.max().item(), err.mean().item())
    assert int(eng.grad.count_nonzero()) == 0
    assert torch.equal(eng.master, m0) and torch.equal(eng.loss, loss0)


def test_sft_trainer_learns_the_responses(tmp_path):
    from distrain_b200 import alignment as al
    from distrain_b200.models.params import ParamLayout, init_flat
    from distrain_b200.utils.checkpoint import load_safetensors
    cfg = _small_cfg()
    tok = al.ByteTokenizer()
    ex = [al.tokenize_conversation(c, tok, "chatml", 256) for c in al.synthetic_conversations(20)]
    c = al.SFTConfig(learning_rate=3e-3, num_epochs=6, batch_size=4, gradient_accumulation_steps=1,
                     max_seq_len=256, warmup_fraction=0.0, log_every_n_steps=5, save_every_n_steps=0,
                     output_dir=str(tmp_path))
    flat = init_flat(ParamLayout(cfg), 0.02, 0)
    tr = al.SFTTrainer(cfg, flat, ex, c, pad_id=tok.pad_id)
    m = tr.train(log=lambda s: None)
    assert m["steps"] == 30 and tr.eng.graph is not None
    assert m["final_loss"] < 0.6 * m["first_loss"], m["history"]
    saved = json.loads(open(os.path.join(tmp_path, "metrics.json")).read())
    assert saved["final_loss"] == m["final_loss"]
    sd = load_safetensors(m["checkpoint"])
    ref = tr.eng.state_dict()
    assert all(torch.equal(sd[k], ref[k]) for k in ref)


def test_dpo_trainer_prefers_the_chosen_response(tmp_path):
    from distrain_b200 import alignment as al
    from distrain_b200.models.params import ParamLayout, init_flat
    cfg = _small_cfg(V=256)
    c = al.DPOConfig(beta=0.1, learning_rate=1e-3, num_epochs=10, batch_size=2, gradient_accumulation_steps=2,
                     max_seq_len=64, warmup_fraction=0.0, log_every_n_steps=1, save_every_n_steps=0,
                     output_dir=str(tmp_path))
    flat = init_flat(ParamLayout(cfg), 0.02, 1)
    tr = al.DPOTrainer(cfg, flat, al.synthetic_preferences(16), c)
    m = tr.train(log=lambda s: None)
    h = m["history"]
    assert m["steps"] == 40
    assert abs(h[0]["loss"] - math.log(2.0)) < 1e-3  # the policy starts as the reference
    assert m["final_reward_accuracy"] == 1.0 and m["final_loss"] < math.log(2.0) - 0.1, h[-1]


def test_lora_sft_trains_adapters_on_frozen_weights(tmp_path):
    """LoRA on the engine: the loss falls, the frozen fp32 weights do not move, the GEMMs' bf16 weights
    are W + s B A, and the saved model is the merged one (adapters saved beside it)."""
    from distrain_b200 import alignment as al
    from distrain_b200.models.params import ParamLayout, init_flat
    from distrain_b200.utils.checkpoint import load_safetensors
    cfg = _small_cfg()
    tok = al.ByteTokenizer()
    ex = [al.tokenize_conversation(c, tok, "chatml", 256) for c in al.synthetic_conversations(20)]
    c = al.SFTConfig(learning_rate=5e-3, num_epochs=6, batch_size=4, gradient_accumulation_steps=1,
                     max_seq_len=256, warmup_fraction=0.0, log_every_n_steps=5, save_every_n_steps=0,
                     output_dir=str(tmp_path), use_lora=True, lora_rank=8, lora_alpha=16.0)
    flat = init_flat(ParamLayout(cfg), 0.02, 0)
    tr = al.SFTTrainer(cfg, flat, ex, c, pad_id=tok.pad_id)
    master0 = tr.eng.master.clone()
    m = tr.train(log=lambda s: None)
    assert m["final_loss"] < 0.9 * m["first_loss"], m["history"]
    assert torch.equal(tr.eng.master, master0)
    lo = tr.lora
    l, name, W, A, B, _, _ = lo.items[0]
    assert B.abs().max().item() > 0
    exact = W + lo.s * B @ A
    err = (tr.eng.wv[l][name].float() - exact).abs()
    assert bool((err <= exact.abs() * 2 ** -8 + 1e-7).all())  # bf16 rounding of W + s B A
    sd = load_safetensors(m["checkpoint"])
    merged = lo.merged_state_dict()
    assert all(torch.equal(sd[k], merged[k]) for k in merged)
    ad = load_safetensors(m["adapter"])
    assert set(ad) == {f"layers.{i}.{t}.lora_{x}" for i in range(cfg.num_layers)
                       for t in ("qkv_w", "o_w", "gu_w", "down_w") for x in "AB"}
    assert m["trainable_params"] == lo.total and tr.eng.m is None
