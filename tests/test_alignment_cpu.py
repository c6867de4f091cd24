"""Post-training data and loss weights (SFT / DPO) on the fp64 oracle model, no GPU.

The engine runs both methods as a cross-entropy backward with per-row weights; these tests pin that the
weights are right: the weighted loss's gradient equals the autograd gradient of the method's own loss."""
import json

import pytest
import torch

from distrain_b200 import alignment as al


def _cfg():
    from distrain_b200.config import ModelConfig
    return ModelConfig(hidden_dim=32, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=64, vocab_size=64,
                       max_seq_len=64, rope_theta=10000.0)


def _params(cfg, seed):
    from distrain_b200.models.params import ParamLayout, init_flat
    L = ParamLayout(cfg)
    flat = init_flat(L, 0.2, seed)
    return {k: v.detach().double().clone().requires_grad_() for k, v in L.views(flat).items()}


def _row_ce(p, cfg, ids):
    """[n, S-1] cross-entropy of predicting token t+1 of every sequence."""
    from distrain_b200.models import oracle
    ids = ids.long()
    z = oracle.logits_fn(p, cfg, ids[:, :-1], mask_value=None)
    lp = torch.log_softmax(z, dim=-1)
    return -lp.gather(-1, ids[:, 1:, None])[..., 0]


def test_templates_mark_assistant_turns():
    tok = al.ByteTokenizer()
    conv = [al.Message("system", "sys"), al.Message("user", "hi"), al.Message("assistant", "hello")]
    for template, trained_text in (("chatml", "hello<|im_end|>\n"), ("zephyr", "hello</s>\n"),
                                   ("llama", " hello </s>")):
        ex = al.tokenize_conversation(conv, tok, template, 512)
        assert len(ex.ids) == len(ex.trained)
        got = tok.decode([i for i, t in zip(ex.ids, ex.trained) if t])
        assert got == trained_text, (template, got)
        text = tok.decode(ex.ids)
        assert "sys" in text and "hi" in text and text.endswith(trained_text)
    llama = tok.decode(al.tokenize_conversation(conv, tok, "llama").ids)
    assert llama.startswith("<s>[INST] <<SYS>>\nsys\n<</SYS>>\n\nhi [/INST]")
    assert tok.decode(al.tokenize_conversation(conv, tok, "chatml").ids).startswith("<|im_start|>system\nsys")
    with pytest.raises(ValueError):
        al.render_chat(conv, "alpaca")
    cut = al.tokenize_conversation(conv, tok, "chatml", max_seq_len=10)
    assert len(cut.ids) == 10 and len(cut.trained) == 10


def test_pack_rows_mask_is_shifted_trained_flags():
    seqs = [[5, 6, 7, 8], [9, 10]]
    trained = [[False, False, True, True], [False, True]]
    ids, mask = al.pack_rows(seqs, trained, seq_len=6, pad_id=0)
    assert ids.tolist() == [[5, 6, 7, 8, 0, 0], [9, 10, 0, 0, 0, 0]]
    # row t predicts token t+1: trained when token t+1 is
    assert mask.tolist() == [[0, 1, 1, 0, 0], [1, 0, 0, 0, 0]]
    w = al.sft_weights(mask)
    assert abs(float(w.sum()) - 1.0) < 1e-7 and float(w[0, 0]) == 0.0


def test_sft_weighted_loss_is_masked_mean():
    cfg = _cfg()
    p = _params(cfg, 1)
    g = torch.Generator().manual_seed(0)
    seqs = [torch.randint(3, 64, (n,), generator=g).tolist() for n in (20, 13, 17)]
    trained = [[j >= n // 2 for j in range(n)] for n in (20, 13, 17)]
    ids, mask = al.pack_rows(seqs, trained, 24, 0)
    ce = _row_ce(p, cfg, ids)
    loss = (al.sft_weights(mask).double() * ce).sum()
    ref = ce[mask.bool()].mean()
    assert abs(loss.item() - ref.item()) < 1e-6 * abs(ref.item())  # fp32 weights


def test_dpo_weights_give_the_dpo_gradient():
    """sum_r w_r * ce_r with the DPO weights (computed from detached log-probabilities) has the same
    gradient as the DPO loss itself, against a reference model that differs from the policy."""
    cfg = _cfg()
    pol, ref_p = _params(cfg, 2), _params(cfg, 3)
    g = torch.Generator().manual_seed(1)
    pairs = []
    for _ in range(3):
        prompt = torch.randint(3, 64, (7,), generator=g).tolist()
        c = prompt + torch.randint(3, 64, (9,), generator=g).tolist()
        r = prompt + torch.randint(3, 64, (5,), generator=g).tolist()
        pairs.append(al.PreferencePair(prompt, c, r))
    ids, mask = al.pair_rows(pairs, 20, 0)
    assert mask[0].sum() == 9 and mask[1].sum() == 5 and mask[0, :6].sum() == 0 and mask[0, 6] == 1
    beta = 0.5
    with torch.no_grad():
        ref_lp = al.sequence_logps(_row_ce(ref_p, cfg, ids), mask)
    # the DPO loss by autograd
    lp = al.sequence_logps(_row_ce(pol, cfg, ids), mask)
    z = beta * ((lp[0::2] - ref_lp[0::2]) - (lp[1::2] - ref_lp[1::2]))
    dpo = torch.nn.functional.softplus(-z).mean()
    dpo.backward()
    want = {k: v.grad.clone() for k, v in pol.items()}
    for v in pol.values():
        v.grad = None
    # the weighted cross-entropy
    w, st = al.dpo_weights(lp.detach(), ref_lp, mask, beta)
    assert abs(st["loss"] - dpo.item()) < 1e-12
    assert st["reward_accuracy"] == float((z > 0).double().mean())
    (w.double() * _row_ce(pol, cfg, ids)).sum().backward()
    for k, v in pol.items():
        # the weights are stored in fp32
        rel = ((v.grad - want[k]).norm() / (want[k].norm() + 1e-30)).item()
        assert rel < 1e-6, (k, rel)


def test_step_order_covers_every_item_each_epoch():
    order = al.step_order(10, 4, 2, seed=3)
    assert len(order) == 6 and all(len(s) == 4 for s in order)
    for e in range(2):
        seen = set(sum(order[3 * e:3 * e + 3], []))
        assert seen == set(range(10))
    with pytest.raises(ValueError):
        al.step_order(0, 4, 1, 0)


def test_synthetic_data_matches_reference_scripts():
    convs = al.synthetic_conversations(7)
    assert len(convs) == 7 and [m.role for m in convs[0]] == ["system", "user", "assistant"]
    assert convs[5][1].content == convs[0][1].content
    pairs = al.synthetic_preferences(3)
    assert pairs[0].prompt_ids == list(range(1, 17))
    assert pairs[0].chosen_ids[16:] == list(range(17, 33)) and pairs[0].rejected_ids[16:] == list(range(33, 49))


def test_jsonl_loaders(tmp_path):
    chat = tmp_path / "chat.jsonl"
    chat.write_text(json.dumps({"messages": [{"role": "user", "content": "q"},
                                             {"role": "assistant", "content": "a"}]}) + "\n\n"
                    + json.dumps({"instruction": "do", "output": "done"}) + "\n")
    convs = al.load_chat_jsonl([str(chat)])
    assert [[m.role for m in c] for c in convs] == [["user", "assistant"]] * 2
    assert convs[1][1].content == "done"
    assert len(al.load_chat_jsonl([str(chat)], max_examples=1)) == 1
    pref = tmp_path / "pref.jsonl"
    pref.write_text(json.dumps({"prompt": "p", "chosen": "good", "rejected": "bad"}) + "\n")
    tok = al.ByteTokenizer()
    (pp,) = al.load_preference_jsonl([str(pref)], tok, "chatml")
    assert pp.chosen_ids[:len(pp.prompt_ids)] == pp.prompt_ids
    assert tok.decode(pp.chosen_ids[len(pp.prompt_ids):]) == "good<|im_end|>\n"
    assert tok.decode(pp.rejected_ids[len(pp.prompt_ids):]) == "bad<|im_end|>\n"
    assert tok.decode(pp.prompt_ids).endswith("<|im_start|>assistant\n")


def test_cli_rejects_missing_data():
    from distrain_b200.cli import main
    with pytest.raises(SystemExit, match="datasets"):
        main(["sft", "--model-size", "micro", "--vocab", "512", "--device", "cpu", "--use-lora"])
    with pytest.raises(SystemExit, match="datasets"):
        main(["dpo", "--model-size", "micro", "--device", "cpu"])


def test_lora_gradients_from_the_weight_gradient():
    """For y = x W_eff^T with W_eff = W + s B A ([N, K], [N, r], [r, K]) the adapters' gradients are
    dA = s B^T dW_eff and dB = s dW_eff A^T, the products the LoRA step forms from the engine's weight
    gradient."""
    torch.manual_seed(0)
    N, K, r, s, M = 24, 40, 4, 2.5, 7
    x = torch.randn(M, K, dtype=torch.float64)
    W = torch.randn(N, K, dtype=torch.float64)
    A = torch.randn(r, K, dtype=torch.float64, requires_grad=True)
    B = torch.randn(N, r, dtype=torch.float64, requires_grad=True)
    t = torch.randn(M, N, dtype=torch.float64)
    loss = lambda Weff: ((x @ Weff.t()).tanh() * t).sum()
    loss(W + s * B @ A).backward()
    Weff = (W + s * B.detach() @ A.detach()).requires_grad_()
    loss(Weff).backward()
    dW = Weff.grad
    assert torch.allclose(A.grad, s * B.detach().t() @ dW, rtol=1e-12, atol=1e-12)
    assert torch.allclose(B.grad, s * dW @ A.detach().t(), rtol=1e-12, atol=1e-12)


def test_lora_tables_merge_and_checkpoint_on_cpu():
    """LoRA bookkeeping without a GPU, on a stand-in engine built from the parameter layout: the AdamW
    chunk tables cover every adapter exactly once (4-aligned starts, one clipping segment per A and per
    B), merge() writes bf16(W + s B A) into the weights the GEMMs read while the fp32 weights stay, and
    the saved model is W + s B A."""
    import types
    from distrain_b200.config import OptimConfig
    from distrain_b200.models.lora import TARGETS, LoraAdapters
    from distrain_b200.models.params import ParamLayout, init_flat
    cfg = _cfg()
    L = ParamLayout(cfg)
    master = init_flat(L, 0.02, 0)
    p16 = master.bfloat16()
    grad = torch.zeros_like(master)
    H, F, d = cfg.hidden_dim, cfg.ffn_hidden_dim, cfg.head_dim()
    W = (cfg.num_heads + 2 * cfg.num_kv_heads) * d
    shp = {"qkv_w": (W, H), "o_w": (H, cfg.num_heads * d), "gu_w": (2 * F, H), "down_w": (H, F)}
    views = lambda buf: [{t: L.group_view(buf, f"layers.{i}.{t}", shp[t]) for t in TARGETS}
                         for i in range(cfg.num_layers)]
    eng = types.SimpleNamespace(tp=None, layout=L, device=torch.device("cpu"), cfg=cfg, optim=OptimConfig(),
                                master=master, p16=p16, gv=views(grad), wv=views(p16), m=None, v=None)
    r = 4
    lo = LoraAdapters(eng, rank=r, alpha=8.0, seed=1)
    assert lo.s == 2.0 and len(lo.items) == cfg.num_layers * len(TARGETS)
    # chunk tables: disjoint, 4-aligned, covering exactly the A and B ranges, one segment each
    covered = torch.zeros(lo.total, dtype=torch.int32)
    for s0, e0 in zip(lo.cstart.tolist(), lo.cend.tolist()):
        assert s0 % 4 == 0 and e0 > s0 and e0 - s0 <= 32768
        covered[s0:e0] += 1
    want = torch.zeros(lo.total, dtype=torch.int32)
    for _, _, Wt, A, B, _, _ in lo.items:
        for t in (A, B):
            off = t.data_ptr() // 4 - lo.p.data_ptr() // 4
            want[off:off + t.numel()] = 1
    assert torch.equal(covered, want)
    assert lo.norms.numel() == 2 * len(lo.items) == int(lo.cseg.max()) + 1
    # merge with non-zero B: bf16 weights of the GEMMs = W + s B A; fp32 weights unchanged
    m0 = master.clone()
    for _, _, _, A, B, _, _ in lo.items:
        B.copy_(torch.randn(B.shape) * 0.1)
    lo.merge()
    assert torch.equal(master, m0)
    for l, name, Wt, A, B, _, _ in lo.items:
        assert torch.equal(eng.wv[l][name], torch.addmm(Wt, B, A, alpha=lo.s).bfloat16())
    sd = lo.merged_state_dict()
    ref = L.to_state_dict(m0)
    changed = [k for k in sd if not torch.equal(sd[k], ref[k])]
    assert changed and all(any(t in k for t in ("q_proj", "k_proj", "v_proj", "o_proj", "gate", "up", "down"))
                           for k in changed), changed
    ad = lo.adapter_state_dict()
    assert len(ad) == 2 * len(lo.items) and ad["layers.0.qkv_w.lora_A"].shape == (r, H)


def test_sft_and_dpo_run_on_the_cpu(tmp_path):
    """The trainers on the CPU engine (fp32 formulation, autograd, the reference AdamW): SFT lowers the
    response loss, DPO starts at log 2 and learns to prefer the chosen continuation, and both write
    their checkpoint and metrics."""
    import math
    from distrain_b200.config import ModelConfig
    from distrain_b200.models.params import ParamLayout, init_flat
    from distrain_b200.utils.checkpoint import load_safetensors
    cfg = ModelConfig(hidden_dim=32, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=64, vocab_size=260,
                      max_seq_len=256, rope_theta=10000.0)
    tok = al.ByteTokenizer()
    ex = [al.tokenize_conversation(c, tok, "zephyr", 96) for c in al.synthetic_conversations(4)]
    c = al.SFTConfig(learning_rate=1e-2, num_epochs=8, batch_size=2, gradient_accumulation_steps=2, max_seq_len=96,
                     warmup_fraction=0.0, log_every_n_steps=1, save_every_n_steps=0,
                     output_dir=str(tmp_path / "sft"))
    tr = al.SFTTrainer(cfg, init_flat(ParamLayout(cfg), 0.05, 0), ex, c, pad_id=tok.pad_id, device="cpu")
    m = tr.train(log=lambda s: None)
    assert m["steps"] == 8 and m["final_loss"] < 0.8 * m["first_loss"], m["history"]
    sd = load_safetensors(m["checkpoint"])
    assert set(sd) == set(ParamLayout(cfg).shapes())
    d = al.DPOConfig(beta=0.5, learning_rate=1e-2, num_epochs=6, batch_size=2, gradient_accumulation_steps=1,
                     max_seq_len=40, warmup_fraction=0.0, log_every_n_steps=1, save_every_n_steps=0,
                     output_dir=str(tmp_path / "dpo"))
    cfg2 = ModelConfig(hidden_dim=32, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=64, vocab_size=64,
                       max_seq_len=64, rope_theta=10000.0)
    dp = al.DPOTrainer(cfg2, init_flat(ParamLayout(cfg2), 0.05, 1), al.synthetic_preferences(4), d, device="cpu")
    m2 = dp.train(log=lambda s: None)
    h = m2["history"]
    assert abs(h[0]["loss"] - math.log(2.0)) < 1e-6
    assert m2["final_reward_accuracy"] == 1.0 and m2["final_loss"] < math.log(2.0), h[-1]
    with pytest.raises(ValueError, match="LoRA"):
        al.SFTTrainer(cfg, init_flat(ParamLayout(cfg), 0.05, 0), ex,
                      al.SFTConfig(use_lora=True, max_seq_len=96, output_dir=str(tmp_path / "x")), device="cpu")


def test_sharegpt_and_conversation_preference_layouts(tmp_path):
    tok = al.ByteTokenizer()
    chat = tmp_path / "hermes.jsonl"
    chat.write_text(json.dumps({"conversations": [{"from": "system", "value": "s"}, {"from": "human", "value": "q"},
                                                  {"from": "gpt", "value": "a"}]}) + "\n")
    (conv,) = al.load_chat_jsonl([str(chat)])
    assert [(m.role, m.content) for m in conv] == [("system", "s"), ("user", "q"), ("assistant", "a")]
    bad = tmp_path / "bad.jsonl"
    bad.write_text(json.dumps({"conversations": [{"from": "robot", "value": "x"}]}) + "\n")
    with pytest.raises(ValueError, match="robot"):
        al.load_chat_jsonl([str(bad)])
    # binarized layout: two conversations sharing a multi-turn context, different last answers
    ctx = [{"role": "user", "content": "hi"}, {"role": "assistant", "content": "hello"},
           {"role": "user", "content": "more"}]
    pref = tmp_path / "pref.jsonl"
    pref.write_text(json.dumps({"chosen": ctx + [{"role": "assistant", "content": "good"}],
                                "rejected": ctx + [{"role": "assistant", "content": "bad"}]}) + "\n"
                    + json.dumps({"prompt": ctx, "chosen": "good", "rejected": "bad"}) + "\n")
    a, b = al.load_preference_jsonl([str(pref)], tok, "chatml")
    assert a == b
    text = tok.decode(a.prompt_ids)
    assert "hello" in text and text.endswith("more<|im_end|>\n<|im_start|>assistant\n")  # earlier answer is context
    assert tok.decode(a.chosen_ids[len(a.prompt_ids):]) == "good<|im_end|>\n"
    assert tok.decode(a.rejected_ids[len(a.prompt_ids):]) == "bad<|im_end|>\n"
    ids, mask = al.pair_rows([a], 256, 0)
    assert int(mask[0].sum()) == len(a.chosen_ids) - len(a.prompt_ids)
