"""Multiple-choice benchmark scoring on the fp32 oracle (CPU): task layouts, the log-likelihood of each
choice against a direct computation, accuracy bookkeeping, and the `evals` command end to end."""
import json

import pytest
import torch

from distrain_b200 import evaluation as ev
from distrain_b200.alignment import ByteTokenizer


def _cfg():
    from distrain_b200.config import ModelConfig
    return ModelConfig(hidden_dim=32, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=64, vocab_size=260,
                       max_seq_len=64, rope_theta=10000.0)


def _flat(cfg, seed=0):
    from distrain_b200.models.params import ParamLayout, init_flat
    return init_flat(ParamLayout(cfg), 0.2, seed)


def test_task_layouts():
    assert ev.normalize_example({"context": "c", "choices": ["a", "b"], "label": 1}) == ("c", ["a", "b"], 1)
    assert ev.normalize_example({"ctx": "c", "endings": ["a", "b", "d"], "label": "2"}) == ("c", ["a", "b", "d"], 2)
    arc = {"question": "q?", "choices": {"text": ["x", "y"], "label": ["A", "B"]}, "answerKey": "B"}
    assert ev.normalize_example(arc) == ("Question: q?\nAnswer:", ["x", "y"], 1)
    assert ev.normalize_example({"question": "q", "choices": ["1", "2", "3", "4"], "answer": "C"})[2] == 2
    assert ev.normalize_example({"question": "q", "choices": ["1", "2"], "answer": 1})[2] == 1
    with pytest.raises(ValueError):
        ev.normalize_example({"text": "x"})


def test_scores_are_the_choice_log_likelihoods():
    """Each score is log p(choice tokens | context) computed directly from the oracle's log-softmax;
    batches are padded and sequences longer than the window lose their left end."""
    from distrain_b200.models import oracle
    from distrain_b200.models.params import ParamLayout
    cfg = _cfg()
    flat = _flat(cfg)
    S = 24
    sc = ev.Scorer(cfg, flat, device="cpu", batch_size=3, seq_len=S)
    g = torch.Generator().manual_seed(0)
    seqs = [torch.randint(3, 259, (n,), generator=g).tolist() for n in (10, 17, 5, 30)]
    starts = [4, 12, 1, 20]
    got = sc.score(seqs, starts)
    p = {k: v.float() for k, v in ParamLayout(cfg).views(flat).items()}
    for s, st, val in zip(seqs, starts, got):
        if len(s) > S:
            st -= len(s) - S
            s = s[-S:]
        ids = torch.tensor([s])
        z = oracle.logits_fn(p, cfg, ids[:, :-1], mask_value=None)
        lp = torch.log_softmax(z.double(), -1)[0]
        want = sum(lp[t - 1, s[t]].item() for t in range(st, len(s)))
        assert abs(val - want) < 1e-6 * max(1.0, abs(want)), (val, want)


def test_accuracy_bookkeeping(tmp_path):
    """A scorer that prefers shorter choices in sum but not per byte separates acc from acc_norm."""
    tok = ByteTokenizer()

    class LenScorer:
        def score(self, seqs, starts):
            return [-(len(s) - st) * 1.0 for s, st in zip(seqs, starts)]
    (tmp_path / "t.jsonl").write_text(json.dumps({"context": "c", "choices": ["aaaa", "b"], "label": 1}) + "\n"
                                      + json.dumps({"context": "c", "choices": ["aaaa", "b"], "label": 0}) + "\n")
    (r,) = ev.evaluate_tasks(LenScorer(), tok, ["t"], str(tmp_path))
    # sum: "b" wins both times (right once); per byte both tie at -1 -> the first choice wins (right once)
    assert r == {"task": "t", "n": 2, "acc": 0.5, "acc_norm": 0.5}
    assert len(ev.load_task(str(tmp_path), "t", limit=1)) == 1


def test_find_checkpoint(tmp_path):
    (tmp_path / "v3").mkdir()
    (tmp_path / "v3" / "model.safetensors").write_bytes(b"x")
    (tmp_path / "v7.safetensors").write_bytes(b"x")
    assert ev.find_checkpoint(str(tmp_path), 3).endswith("v3/model.safetensors")
    assert ev.find_checkpoint(str(tmp_path), 7).endswith("v7.safetensors")
    with pytest.raises(FileNotFoundError):
        ev.find_checkpoint(str(tmp_path), 5)


def test_evals_command_on_versions(tmp_path, capsys):
    from distrain_b200.cli import main
    from distrain_b200.models.params import ParamLayout
    from distrain_b200.utils.checkpoint import save_safetensors
    cfg = _cfg()
    L = ParamLayout(cfg)
    for v in (1, 2):
        (tmp_path / "ck" / f"v{v}").mkdir(parents=True)
        save_safetensors(L.to_state_dict(_flat(cfg, v)), str(tmp_path / "ck" / f"v{v}" / "model.safetensors"))
    tasks = tmp_path / "tasks"
    tasks.mkdir()
    (tasks / "hellaswag.jsonl").write_text("".join(
        json.dumps({"ctx": f"c{i}", "endings": ["x", "yy", "zzz"], "label": i % 3}) + "\n" for i in range(5)))
    main(["evals", "--checkpoint-dir", str(tmp_path / "ck"), "--versions", "1,2,9", "--quick", "--device", "cpu",
          "--task-dir", str(tasks), "--seq-len", "32", "--batch-size", "4", "--output-dir", str(tmp_path / "out")])
    lines = [json.loads(x) for x in capsys.readouterr().out.strip().splitlines()]
    assert [x["version"] for x in lines] == [1, 2]
    for v in (1, 2):
        saved = json.loads((tmp_path / "out" / f"v{v}.json").read_text())
        (r,) = saved["results"]
        assert r["task"] == "hellaswag" and r["n"] == 5 and 0.0 <= r["acc"] <= 1.0


def test_piqa_and_winogrande_layouts(tmp_path):
    ctxs, conts, label = ev.example_pairs({"goal": "g", "sol1": "a", "sol2": "b", "label": 1})
    assert ctxs == ["Question: g\nAnswer:"] * 2 and conts == [" a", " b"] and label == 1
    ctxs, conts, label = ev.example_pairs({"sentence": "The cup fell because _ was slippery.", "option1": "the cup",
                                           "option2": "the table", "answer": "2"})
    assert ctxs == ["The cup fell because the cup", "The cup fell because the table"]
    assert conts == [" was slippery."] * 2 and label == 1
    # scoring: each option is judged by the log-likelihood of the shared remainder in its own context
    tok = ByteTokenizer()

    class PrefersTable:
        def score(self, seqs, starts):
            return [0.0 if "table" in tok.decode(s[:st]) else -1.0 for s, st in zip(seqs, starts)]
    (tmp_path / "winogrande.jsonl").write_text(json.dumps(
        {"sentence": "It fell off _ today.", "option1": "the cup", "option2": "the table", "answer": "2"}) + "\n")
    (r,) = ev.evaluate_tasks(PrefersTable(), tok, ["winogrande"], str(tmp_path))
    assert r["acc"] == 1.0 and r["n"] == 1
