"""Benchmark scoring on the CUDA engine's forward-only loss pass against the fp32 oracle scorer."""
import json

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_engine_scores_match_oracle(tmp_path):
    from distrain_b200 import evaluation as ev
    from distrain_b200.alignment import ByteTokenizer
    from distrain_b200.config import ModelConfig
    from distrain_b200.models.params import ParamLayout, init_flat
    cfg = ModelConfig(hidden_dim=128, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=256, vocab_size=512,
                      max_seq_len=128, rope_theta=10000.0)
    flat = init_flat(ParamLayout(cfg), 0.05, 3)
    g = torch.Generator().manual_seed(1)
    seqs = [torch.randint(3, 259, (n,), generator=g).tolist() for n in (40, 65, 9, 100, 64, 12, 77)]
    starts = [10, 30, 2, 90, 1, 11, 40]
    gpu = ev.Scorer(cfg, flat, device="cuda:0", batch_size=4, seq_len=65).score(seqs, starts)
    cpu = ev.Scorer(cfg, flat, device="cpu", batch_size=4, seq_len=65).score(seqs, starts)
    for a, b, s, st in zip(gpu, cpu, seqs, starts):
        n = min(len(s), 65) - max(st - max(len(s) - 65, 0), 1)
        assert abs(a - b) < 0.02 * n + 0.05, (a, b, n)
    # the same through the command's entry point on a task file
    (tmp_path / "arc_easy.jsonl").write_text("".join(json.dumps(
        {"question": f"q{i}", "choices": {"text": ["a", "bb"], "label": ["A", "B"]}, "answerKey": "AB"[i % 2]}) + "\n"
        for i in range(6)))
    r_gpu = ev.evaluate_tasks(ev.Scorer(cfg, flat, "cuda:0", 4, 65), ByteTokenizer(), ["arc_easy"], str(tmp_path))
    r_cpu = ev.evaluate_tasks(ev.Scorer(cfg, flat, "cpu", 4, 65), ByteTokenizer(), ["arc_easy"], str(tmp_path))
    assert r_gpu[0]["n"] == 6 and abs(r_gpu[0]["acc"] - r_cpu[0]["acc"]) <= 1 / 6 + 1e-9


def test_inference_engine_matches_training_engine():
    """The forward-only engine (no gradients, optimizer state or backward scratch; one set of block
    buffers) gives the training engine's per-row losses bit for bit and refuses a backward."""
    from distrain_b200.config import ModelConfig
    from distrain_b200.models.engine import TrainEngine
    from distrain_b200.models.params import ParamLayout, init_flat
    cfg = ModelConfig(hidden_dim=128, num_layers=3, num_heads=4, num_kv_heads=2, ffn_hidden_dim=256, vocab_size=512,
                      max_seq_len=128, rope_theta=10000.0)
    flat = init_flat(ParamLayout(cfg), 0.05, 4)
    tokens = torch.randint(0, 512, (4, 65), dtype=torch.int32).cuda()
    full = TrainEngine(cfg, 4, 65, device="cuda", flat_init=flat)
    inf = TrainEngine(cfg, 4, 65, device="cuda", flat_init=flat, inference=True)
    assert inf.grad is None and inf.m is None and inf.dgu is None and inf.qkv[0] is inf.qkv[2]
    full.set_tokens(tokens)
    inf.set_tokens(tokens)
    a = full.forward_loss(0).clone()
    b = inf.forward_loss(0).clone()
    assert torch.equal(a, b)
    with pytest.raises(RuntimeError):
        inf.forward_backward()


def test_held_out_loss_on_the_engine():
    """cli eval's loss on a GPU (forward-only engine) against the fp32 formulation on the CPU."""
    from distrain_b200.cli import _eval_loss
    from distrain_b200.config import ModelConfig
    from distrain_b200.models.params import ParamLayout, init_flat
    cfg = ModelConfig(hidden_dim=128, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=256, vocab_size=512,
                      max_seq_len=128, rope_theta=10000.0)
    L = ParamLayout(cfg)
    sd = L.to_state_dict(init_flat(L, 0.05, 6))
    g = torch.Generator().manual_seed(2)
    batches = [torch.randint(0, 512, (3, 65), generator=g, dtype=torch.int32) for _ in range(2)]
    gpu = _eval_loss(sd, cfg, batches, "cuda:0")
    cpu = _eval_loss(sd, cfg, batches, "cpu")
    assert abs(gpu - cpu) < 5e-3, (gpu, cpu)
