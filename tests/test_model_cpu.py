"""CPU tests: presets, flat layout, oracle model semantics (reference model.rs tests, restated)."""
import math

import pytest
import torch

from distrain_b200.config import preset, ModelConfig, bench_config, cosine_lr, CoordinatorConfig, RunConfig
from distrain_b200.models.params import ParamLayout, init_flat
from distrain_b200.models import oracle


def test_presets_match_reference_table():
    t = preset("tiny")
    assert (t.hidden_dim, t.num_layers, t.num_heads, t.num_kv_heads, t.ffn_hidden_dim) == (768, 12, 12, 4, 2048)
    assert 100_000_000 < t.param_count() < 150_000_000
    assert preset("medium").head_dim() == 128 and preset("medium").num_gqa_groups() == 4
    m = preset("micro-test")
    assert (m.vocab_size, m.max_seq_len, m.rope_theta) == (256, 64, 500_000.0)
    for n in ("125m", "1b", "7b", "13b", "small", "large"):
        c = preset(n)
        assert c.param_count() > 0 and c.head_dim() > 0 and c.num_gqa_groups() >= 1
    with pytest.raises(KeyError):
        preset("nope")


def test_bench_configs():
    m = bench_config("micro")
    assert (m.model.vocab_size, m.seq_len, m.model.rope_theta, m.micro_batch, m.push_every) == (32768, 128, 1e4, 4, 20)
    t = bench_config("tiny")
    assert (t.seq_len, t.micro_batch, t.push_every, t.compression.top_k_fraction) == (1024, 32, 50, 0.10)
    l = bench_config("large")
    assert l.tp == 2 and l.activation_checkpointing


def test_layout_names_and_contiguous_groups():
    cfg = preset("micro")
    L = ParamLayout(cfg)
    names = [e.name for e in L.entries]
    assert names[0] == "embedding.embedding.weight" and "final_norm.weight" in names
    assert L.num_params() == cfg.param_count() + 1  # + output_scale, which the reference formula omits
    q = L.by_name["layers.0.attention.q_proj.weight"]
    k = L.by_name["layers.0.attention.k_proj.weight"]
    v = L.by_name["layers.0.attention.v_proj.weight"]
    assert k.offset == q.offset + q.numel and v.offset == k.offset + k.numel
    g = L.by_name["layers.1.ffn.gate_proj.weight"]
    u = L.by_name["layers.1.ffn.up_proj.weight"]
    assert u.offset == g.offset + g.numel
    for s, e in L.groups.values():
        assert s % 64 == 0
    flat = init_flat(L, 0.02, 0)
    sd = L.to_state_dict(flat)
    flat2 = torch.zeros_like(flat)
    L.load_state_dict(flat2, sd)
    assert torch.equal(flat, flat2)
    assert sd["layers.0.attn_norm.weight"].eq(1).all() and sd["embedding.output_scale"].item() == 1.0


def test_chunk_tables_cover_every_param():
    L = ParamLayout(preset("micro"))
    seg, st, en, n = L.chunk_tables("cpu", chunk=1000)
    covered = torch.zeros(L.total, dtype=torch.bool)
    for s, e in zip(st.tolist(), en.tolist()):
        covered[s:e] = True
    for e in L.entries:
        assert covered[e.offset:e.offset + e.numel].all()
    assert n == len(L.entries)


def test_oracle_forward_and_loss():
    cfg = bench_config("micro").model
    cfg.vocab_size = 256
    L = ParamLayout(cfg)
    p = L.views(init_flat(L, 0.02, 0))
    tokens = torch.randint(0, 256, (2, 17))
    loss = oracle.lm_loss(p, cfg, tokens)
    assert loss.item() > 0 and abs(loss.item() - math.log(256)) < 0.5
    z = oracle.logits_fn(p, cfg, tokens[:, :-1])
    assert z.shape == (2, 16, 256)
    # -1e4 additive mask and exact -inf mask agree
    l2 = oracle.lm_loss(p, cfg, tokens, mask_value=None)
    assert abs(l2.item() - loss.item()) < 1e-5


def test_rope_tables_reference_formula():
    cfg = ModelConfig(hidden_dim=64, num_heads=4, rope_theta=500000.0)
    cos, sin = oracle.rope_tables(cfg, 8)
    d = 16
    i = 3
    f = 1.0 / (500000.0 ** (2 * i / d))
    assert abs(cos[5, i].item() - math.cos(5 * f)) < 1e-5


def test_cosine_lr_reference_values():
    assert cosine_lr(0, 10, 100, 1.0, 0.0) == 0.0
    assert abs(cosine_lr(10, 10, 100, 1.0, 0.0) - 1.0) < 1e-12
    assert abs(cosine_lr(100, 10, 100, 1.0, 0.1) - 0.1) < 1e-12
    assert abs(cosine_lr(55, 10, 100, 1.0, 0.0) - 0.5) < 1e-12


def test_adamw_ref_per_tensor_clip():
    p = {"a": torch.zeros(4, requires_grad=False), "b": torch.zeros(2)}
    opt = oracle.AdamWRef(p, lr=0.1, weight_decay=0.0, clip=1.0)
    p["a"].grad = torch.tensor([3.0, 4.0, 0.0, 0.0])
    p["b"].grad = torch.tensor([0.1, 0.0])
    opt.step()
    # first step of Adam moves each coordinate by ~lr * sign(g)
    assert torch.allclose(p["a"][:2], torch.tensor([-0.1, -0.1]), atol=1e-3)
    assert abs(p["b"][0].item() + 0.1) < 1e-3


def test_coordinator_env_mapping():
    c = CoordinatorConfig.from_env({"PORT": "9001", "MIN_CONTRIBUTIONS": "3", "OUTER_LR": "1.0",
                                    "R2_BUCKET": "b", "S3_EXTERNAL_ENDPOINT": "http://x:9000"})
    assert (c.port, c.min_contributions, c.outer_lr, c.storage.bucket) == (9001, 3, 1.0, "b")
    assert c.external_storage_endpoint == "http://x:9000"
    r = RunConfig.from_json(bench_config("tiny").to_json())
    assert r.model.hidden_dim == 768 and r.compression.int8_block == 256
