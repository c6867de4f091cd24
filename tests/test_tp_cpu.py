"""Tensor-parallel helpers on the CPU: shard / gather round trip, per-segment clip-norm weights, and a
sharded layout whose local shapes match the shards of a full state dict."""
import torch

from distrain_b200.config import ModelConfig
from distrain_b200.models.params import ParamLayout, init_flat
from distrain_b200.parallel.tensor_parallel import shard_state_dict, gather_state_dict, split_dim, norm_weights


def _cfg():
    return ModelConfig(hidden_dim=128, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=256, vocab_size=512)


def test_split_rules():
    assert split_dim("layers.0.attention.q_proj.weight") == 0
    assert split_dim("layers.0.attention.k_proj.bias") == 0
    assert split_dim("layers.0.attention.o_proj.weight") == 1
    assert split_dim("layers.0.ffn.gate_proj.weight") == 0
    assert split_dim("layers.0.ffn.down_proj.weight") == 1
    for name in ("embedding.embedding.weight", "embedding.output_scale", "final_norm.weight",
                 "layers.1.attn_norm.weight", "layers.1.ffn_norm.weight"):
        assert split_dim(name) is None


def test_shard_gather_roundtrip_and_local_layout():
    cfg = _cfg()
    full = ParamLayout(cfg)
    sd = full.to_state_dict(init_flat(full, 0.02, 7))
    shards = [shard_state_dict(sd, cfg, r, 2) for r in range(2)]
    back = gather_state_dict(shards)
    assert set(back) == set(sd)
    for k in sd:
        assert torch.equal(back[k], sd[k]), k
    for r in range(2):
        loc = ParamLayout(cfg, r, 2)
        flat = torch.zeros(loc.total)
        loc.load_state_dict(flat, shards[r])  # shapes must line up with the local layout
        assert loc.num_params() == sum(v.numel() for v in shards[r].values())
    # the local layouts together hold every split parameter exactly once, replicated ones twice
    n_split = sum(v.numel() for k, v in sd.items() if split_dim(k) is not None)
    n_rep = sum(v.numel() for k, v in sd.items() if split_dim(k) is None)
    assert sum(ParamLayout(cfg, r, 2).num_params() for r in range(2)) == n_split + 2 * n_rep


def test_norm_weights_sum_to_full_norm():
    cfg = _cfg()
    full = ParamLayout(cfg)
    g = torch.randn(full.total)
    sd = full.to_state_dict(g)
    want = torch.tensor([float((sd[e.name].double() ** 2).sum()) for e in full.entries], dtype=torch.float64)
    got = torch.zeros(len(full.entries), dtype=torch.float64)
    for r in range(2):
        loc = ParamLayout(cfg, r, 2)
        w = norm_weights(loc, "cpu").double()
        sh = shard_state_dict(sd, cfg, r, 2)
        local = torch.tensor([float((sh[e.name].double() ** 2).sum()) for e in loc.entries], dtype=torch.float64)
        got += local * w
    assert torch.allclose(got, want, rtol=1e-9)
