"""In-box checkpoint persistence on the host side: the writer stores the reference layout with
retention, the newest version is found by scanning the store, resume reads it back, and per-shard files
of a tensor-parallel node gather into the reference state dict."""
import torch

from distrain_b200 import protocol as P
from distrain_b200.config import ModelConfig
from distrain_b200.models.params import ParamLayout, init_flat
from distrain_b200.parallel.inbox_ckpt import (CheckpointWriter, gather_checkpoint, latest_version, resume_flat,
                                               shard_checkpoint_path, stored_versions)
from distrain_b200.parallel.tensor_parallel import shard_state_dict
from distrain_b200.utils.checkpoint import load_safetensors_bytes
from distrain_b200.utils.storage import FsStore


def _cfg():
    return ModelConfig(hidden_dim=64, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=128, vocab_size=256)


def test_writer_retention_and_resume(tmp_path):
    cfg = _cfg()
    L = ParamLayout(cfg)
    store = FsStore(str(tmp_path))
    w = CheckpointWriter(store, L, every=2, keep_versions=2)
    flats = {}
    for v in range(1, 9):
        f = init_flat(L, 0.02, seed=v)
        flats[v] = f
        if w.due(v):
            w.snapshot(f, v, meta={"contributions_accepted": 3})
    w.close()
    assert stored_versions(store) == [6, 8]
    assert latest_version(store) == 8
    assert store.get_json(P.checkpoint_metadata_path(8))["version"] == 8
    back = resume_flat(store, L, 8)
    for e in L.entries:
        assert torch.equal(back[e.offset:e.offset + e.numel], flats[8][e.offset:e.offset + e.numel])
    sd = load_safetensors_bytes(store.get(P.checkpoint_path(8)))
    assert set(sd) == {e.name for e in L.entries}


def test_tensor_parallel_shard_files_gather(tmp_path):
    cfg = _cfg()
    full = ParamLayout(cfg)
    flat = init_flat(full, 0.02, seed=1)
    ref = full.to_state_dict(flat)
    store = FsStore(str(tmp_path))
    for t in range(2):
        L = ParamLayout(cfg, t, 2)
        lf = torch.zeros(L.total)
        L.load_state_dict(lf, shard_state_dict(ref, cfg, t, 2))
        w = CheckpointWriter(store, L, every=1, keep_versions=5, shard=t, n_shards=2)
        w.snapshot(lf, 4)
        w.close()
    assert store.exists(shard_checkpoint_path(4, 1, 2)) and latest_version(store, 2) == 4
    got = gather_checkpoint(store, 4, 2)
    for k in ref:
        assert torch.equal(got[k], ref[k]), k


def test_export_hf_from_tensor_parallel_shard_files(tmp_path):
    """export-hf --store --tp 2 gathers the shard files of the newest version and writes a Hugging Face
    directory whose weights are the full model's."""
    import json
    from distrain_b200 import cli
    from distrain_b200.utils.checkpoint import load_safetensors
    cfg = _cfg()
    full = ParamLayout(cfg)
    ref = full.to_state_dict(init_flat(full, 0.02, seed=3))
    store = FsStore(str(tmp_path / "st"))
    for t in range(2):
        L = ParamLayout(cfg, t, 2)
        lf = torch.zeros(L.total)
        L.load_state_dict(lf, shard_state_dict(ref, cfg, t, 2))
        w = CheckpointWriter(store, L, every=1, keep_versions=5, shard=t, n_shards=2)
        w.snapshot(lf, 6)
        w.close()
    cli.main(["export-hf", "--store", str(tmp_path / "st"), "--tp", "2", str(tmp_path / "hf")])
    hf = load_safetensors(str(tmp_path / "hf" / "model.safetensors"))
    assert torch.equal(hf["model.layers.0.mlp.gate_proj.weight"], ref["layers.0.ffn.gate_proj.weight"])
    assert torch.equal(hf["model.embed_tokens.weight"], ref["embedding.embedding.weight"])
    assert json.loads((tmp_path / "hf" / "config.json").read_text())["num_hidden_layers"] == cfg.num_layers
