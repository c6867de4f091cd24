"""Multiple-choice benchmark evaluation of checkpoints by log-likelihood scoring, offline.

Counterpart of the reference's ``scripts/run_evals.py``, whose ``distrain.eval.benchmarks`` module is not
in its repository (``run_evals.py:29-39``). The script's surface is kept: one checkpoint, ``random`` (an
untrained model of ``--model-size``), or ``--checkpoint-dir`` with ``--versions`` (``v{n}/model.safetensors``,
``step_{n}/model.safetensors`` or ``v{n}.safetensors``, ``run_evals.py:43-54``); ``--tasks`` or
``--quick``; ``--limit``; ``--batch-size``; one JSON result per checkpoint in ``--output-dir`` and a
summary table. Task data are local JSONL files (``<task-dir>/<task>.jsonl``) in place of hub downloads:
one example per line, in the generic form ``{"context", "choices", "label"}`` or in the field layouts of
the usual sources (HellaSwag: ctx / endings / label; ARC: question / choices{text, label} / answerKey;
MMLU: question / choices / answer; PIQA: goal / sol1 / sol2 / label; Winogrande: sentence / option1 /
option2 / answer, scored by the sentence's remainder after each option fills its blank).

Scoring follows the usual log-likelihood protocol: each choice is appended, after a space, to the
context and scored by the sum of its tokens' log-probabilities; ``acc`` is the argmax of that sum,
``acc_norm`` the argmax of the sum divided by the choice's length in UTF-8 bytes. On a GPU the
sequences go through ``TrainEngine.forward_loss`` (the CUDA forward and the fused LM-head
cross-entropy, a batch at a time); on the CPU through the fp32 oracle.
"""
from __future__ import annotations

import json
import os
import time
from typing import Dict, List, Optional, Sequence, Tuple

import torch

QUICK_TASKS = ["hellaswag"]
FULL_TASKS = ["mmlu", "hellaswag", "arc_challenge", "arc_easy"]


def normalize_example(r: dict) -> Tuple[str, List[str], int]:
    """(context, choices, index of the correct choice) of one task line."""
    if "context" in r and "choices" in r:
        return r["context"], list(r["choices"]), int(r["label"])
    if "ctx" in r and "endings" in r:  # HellaSwag
        return r["ctx"], list(r["endings"]), int(r["label"])
    if "question" in r and isinstance(r.get("choices"), dict):  # ARC
        labels = list(r["choices"]["label"])
        return f"Question: {r['question']}\nAnswer:", list(r["choices"]["text"]), labels.index(r["answerKey"])
    if "question" in r and "choices" in r and "answer" in r:  # MMLU
        a = r["answer"]
        return f"{r['question']}\nAnswer:", list(r["choices"]), "ABCDEFGH".index(a) if isinstance(a, str) else int(a)
    if "goal" in r and "sol1" in r:  # PIQA
        return f"Question: {r['goal']}\nAnswer:", [r["sol1"], r["sol2"]], int(r["label"])
    raise ValueError(f"unrecognised task line (keys {sorted(r)})")


def example_pairs(r: dict) -> Tuple[List[str], List[str], int]:
    """(context per choice, scored continuation per choice, correct index) of one task line. Most layouts
    share one context and score " " + choice; Winogrande (sentence with a blank "_", option1 / option2,
    answer "1" / "2") puts each option into the blank and scores the rest of the sentence after it."""
    if "sentence" in r and "option1" in r:
        i = r["sentence"].index("_")
        before, after = r["sentence"][:i], r["sentence"][i + 1:]
        opts = [r["option1"], r["option2"]]
        return [before + o for o in opts], [after] * 2, int(r["answer"]) - 1
    ctx, choices, label = normalize_example(r)
    return [ctx] * len(choices), [" " + c for c in choices], label


def load_task(task_dir: str, task: str, limit: Optional[int] = None) -> List[Tuple[List[str], List[str], int]]:
    """``example_pairs`` of the first ``limit`` lines of ``<task_dir>/<task>.jsonl``."""
    path = os.path.join(task_dir, f"{task}.jsonl")
    out = []
    with open(path) as f:
        for line in f:
            if line.strip():
                out.append(example_pairs(json.loads(line)))
                if limit is not None and len(out) >= limit:
                    break
    return out


def find_checkpoint(checkpoint_dir: str, version: int) -> str:
    for c in (os.path.join(checkpoint_dir, f"v{version}", "model.safetensors"),
              os.path.join(checkpoint_dir, f"step_{version}", "model.safetensors"),
              os.path.join(checkpoint_dir, f"v{version}.safetensors")):
        if os.path.exists(c):
            return c
    raise FileNotFoundError(f"no checkpoint for version {version} in {checkpoint_dir}")


class Scorer:
    """Sum of the log-probabilities of each sequence's target span, a batch at a time: the CUDA engine's
    forward-only loss pass on a GPU, the fp32 oracle on the CPU."""

    def __init__(self, cfg, flat: torch.Tensor, device: str = "cuda:0", batch_size: int = 8, seq_len: int = 512,
                 pad_id: int = 0):
        from .models.params import ParamLayout
        self.cfg, self.B, self.S, self.pad = cfg, batch_size, seq_len, pad_id
        cfg.max_seq_len = max(cfg.max_seq_len, seq_len)
        self.dev = torch.device(device)
        if self.dev.type == "cuda":
            from .models.engine import TrainEngine
            self.eng = TrainEngine(cfg, batch_size, seq_len, device=device, flat_init=flat, inference=True)
        else:
            self.eng = None
            self.params = {k: v.float() for k, v in ParamLayout(cfg).views(flat).items()}

    def _row_ce(self, ids: torch.Tensor) -> torch.Tensor:
        if self.eng is not None:
            self.eng.set_tokens(ids.to(self.dev))
            return self.eng.forward_loss(0).view(self.B, self.S - 1).double().cpu()
        from .models import oracle
        with torch.no_grad():
            z = oracle.logits_fn(self.params, self.cfg, ids[:, :-1].long(), mask_value=None)
            lp = torch.log_softmax(z.double(), dim=-1)
            return -lp.gather(-1, ids[:, 1:, None].long())[..., 0]

    def score(self, seqs: Sequence[Sequence[int]], starts: Sequence[int]) -> List[float]:
        """log p(seq[start:] | seq[:start]) per sequence. Sequences longer than the window lose tokens on
        the left; the first token of the window is never a target."""
        from .alignment import pack_rows
        out: List[float] = []
        for i in range(0, len(seqs), self.B):
            chunk, trained = [], []
            for s, st in zip(seqs[i:i + self.B], starts[i:i + self.B]):
                s = list(s)
                if len(s) > self.S:
                    st -= len(s) - self.S
                    s = s[-self.S:]
                chunk.append(s)
                trained.append([j >= max(st, 1) for j in range(len(s))])
            n = len(chunk)
            chunk += [[]] * (self.B - n)
            trained += [[]] * (self.B - n)
            ids, mask = pack_rows(chunk, trained, self.S, self.pad)
            lp = -(self._row_ce(ids) * mask.double()).sum(-1)
            out += lp[:n].tolist()
        return out


def evaluate_tasks(scorer: Scorer, tok, tasks: Sequence[str], task_dir: str, limit: Optional[int] = None
                   ) -> List[Dict]:
    results = []
    for task in tasks:
        examples = load_task(task_dir, task, limit)
        seqs, starts, nbytes, spans = [], [], [], []
        for ctxs, conts, _ in examples:
            spans.append((len(seqs), len(conts)))
            for ctx, cont in zip(ctxs, conts):
                c, t = tok.encode(ctx), tok.encode(cont)
                seqs.append(c + t)
                starts.append(len(c))
                nbytes.append(max(len(cont.encode("utf-8")), 1))
        lps = scorer.score(seqs, starts)
        acc = acc_norm = 0
        for (first, k), (_, _, label) in zip(spans, examples):
            lp = lps[first:first + k]
            acc += int(max(range(k), key=lambda j: lp[j]) == label)
            acc_norm += int(max(range(k), key=lambda j: lp[j] / nbytes[first + j]) == label)
        n = max(len(examples), 1)
        results.append({"task": task, "n": len(examples), "acc": acc / n, "acc_norm": acc_norm / n})
    return results


def evaluate_checkpoint(checkpoint: str, tasks: Sequence[str], task_dir: str, model_size: str = "125m",
                        device: str = "cuda:0", batch_size: int = 8, seq_len: int = 512, limit: Optional[int] = None,
                        tokenizer: Optional[str] = None, version: Optional[int] = None, vocab: Optional[int] = None,
                        seed: int = 0) -> Dict:
    """Scores of one checkpoint (a safetensors path, or ``random`` for an untrained model)."""
    from .alignment import ByteTokenizer, FileTokenizer
    from .models.params import ParamLayout, init_flat
    if checkpoint == "random":
        from .cli import _model_cfg
        cfg = _model_cfg(model_size, vocab=vocab)
        flat = init_flat(ParamLayout(cfg), seed=seed)
    else:
        from .cli import _infer_model_config
        from .utils.checkpoint import load_safetensors
        sd = load_safetensors(checkpoint)
        cfg = _infer_model_config(sd)
        L = ParamLayout(cfg)
        flat = torch.zeros(L.total)
        L.load_state_dict(flat, sd)
    tok = FileTokenizer(tokenizer) if tokenizer else ByteTokenizer()
    if tok.vocab_size > cfg.vocab_size:
        raise ValueError(f"tokenizer vocabulary {tok.vocab_size} > model vocabulary {cfg.vocab_size}")
    t0 = time.perf_counter()
    scorer = Scorer(cfg, flat, device, batch_size, seq_len, tok.pad_id)
    res = evaluate_tasks(scorer, tok, tasks, task_dir, limit)
    return {"checkpoint": checkpoint, "version": version, "results": res,
            "seconds": round(time.perf_counter() - t0, 3)}


def summary_table(result: Dict) -> str:
    rows = [f"{'task':<16} {'n':>6} {'acc':>8} {'acc_norm':>9}"]
    for r in result["results"]:
        rows.append(f"{r['task']:<16} {r['n']:>6} {r['acc']:>8.4f} {r['acc_norm']:>9.4f}")
    head = result["checkpoint"] + (f" (version {result['version']})" if result["version"] is not None else "")
    return head + "\n" + "\n".join(rows)


def save_result(result: Dict, output_dir: str) -> str:
    os.makedirs(output_dir, exist_ok=True)
    name = (f"v{result['version']}" if result["version"] is not None
            else os.path.splitext(os.path.basename(result["checkpoint"]))[0] or "checkpoint")
    path = os.path.join(output_dir, f"{name}.json")
    with open(path, "w") as f:
        json.dump(result, f, indent=2)
    return path
