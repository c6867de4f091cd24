"""Checkpoint export to the Hugging Face Qwen2 layout: transformers loads the exported directory and its
logits match the fp32 oracle's (causal mask with -inf, the output scale folded into the final norm),
with and without q/k/v bias; the export-hf command writes the same files."""
import json

import pytest
import torch

from distrain_b200 import cli
from distrain_b200.config import preset
from distrain_b200.models import oracle
from distrain_b200.models.params import ParamLayout, init_flat
from distrain_b200.utils.checkpoint import save_safetensors
from distrain_b200.utils.hf_export import export_hf

transformers = pytest.importorskip("transformers")


def _weights(cfg, seed):
    L = ParamLayout(cfg)
    sd = L.to_state_dict(init_flat(L, 0.05, seed))
    g = torch.Generator().manual_seed(seed)
    for k, v in sd.items():
        if k.endswith("norm.weight") or k.endswith(".bias"):
            sd[k] = 1.0 + 0.1 * torch.randn(v.shape, generator=g) if k.endswith("weight") else \
                0.05 * torch.randn(v.shape, generator=g)
    sd["embedding.output_scale"] = torch.full_like(sd["embedding.output_scale"], 1.7)
    return sd


@pytest.mark.parametrize("bias", [True, False])
def test_exported_model_matches_the_oracle(tmp_path, bias):
    cfg = preset("micro")
    cfg.qkv_bias = bias
    sd = _weights(cfg, 3)
    export_hf(sd, cfg, str(tmp_path / "hf"))
    m = transformers.AutoModelForCausalLM.from_pretrained(str(tmp_path / "hf"), attn_implementation="eager",
                                                          dtype=torch.float32)
    m.eval()
    ids = torch.randint(0, cfg.vocab_size, (2, 24), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        got = m(input_ids=ids).logits
        want = oracle.logits_fn(sd, cfg, ids, mask_value=None)
    assert torch.allclose(got, want, atol=2e-4, rtol=1e-4), float((got - want).abs().max())


def test_export_command(tmp_path, capsys):
    cfg = preset("micro")
    sd = _weights(cfg, 4)
    ck = tmp_path / "model.safetensors"
    ck.write_bytes(save_safetensors(sd))
    cli.main(["export-hf", str(ck), str(tmp_path / "out"), "--max-seq-len", "256"])
    rec = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert rec["event"] == "exported_hf"
    conf = json.loads((tmp_path / "out" / "config.json").read_text())
    assert (conf["num_attention_heads"], conf["num_key_value_heads"], conf["max_position_embeddings"]) == (4, 2, 256)
    assert (tmp_path / "out" / "model.safetensors").stat().st_size > 0


def test_import_roundtrip_and_bootstrap_from_hf(tmp_path, capsys):
    """Export -> import gives a model with the same logits (output scale now inside the final norm), and
    bootstrap --from-hf writes it as checkpoint v0."""
    from distrain_b200.utils.checkpoint import load_safetensors_bytes
    from distrain_b200.utils.hf_export import from_hf
    from distrain_b200.utils.storage import FsStore
    from distrain_b200 import protocol as P
    cfg = preset("micro")
    sd = _weights(cfg, 6)
    export_hf(sd, cfg, str(tmp_path / "hf"))
    back, cfg2 = from_hf(str(tmp_path / "hf"))
    assert (cfg2.num_heads, cfg2.num_kv_heads, cfg2.hidden_dim, cfg2.rope_theta) == \
        (cfg.num_heads, cfg.num_kv_heads, cfg.hidden_dim, cfg.rope_theta)
    ids = torch.randint(0, cfg.vocab_size, (2, 20), generator=torch.Generator().manual_seed(2))
    assert torch.allclose(oracle.logits_fn(back, cfg2, ids), oracle.logits_fn(sd, cfg, ids), atol=1e-5, rtol=1e-5)
    cli.main(["bootstrap", "--store", str(tmp_path / "store"), "--from-hf", str(tmp_path / "hf")])
    v0 = load_safetensors_bytes(FsStore(str(tmp_path / "store")).get(P.checkpoint_path(0)))
    assert all(torch.equal(v0[k], back[k]) for k in back)
