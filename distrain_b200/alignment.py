"""Post-training on the CUDA training engine: supervised fine-tuning (SFT) with the loss on assistant
tokens only, and direct preference optimisation (DPO).

The reference ships both as command-line scripts whose trainer package is not in its repository
(``scripts/run_sft.py:33-44`` imports ``distrain.alignment.{chat_template,data,sft}``,
``scripts/run_dpo.py:28-35`` imports ``distrain.alignment.{dpo,preference_data}``). Their command
lines and behaviour are kept: base / SFT checkpoint or a random model of a preset size, chat template
(chatml / llama / zephyr), synthetic data (``run_sft.py:52-83``: five system / user / assistant
conversations; ``run_dpo.py:40-55``: a 16-token prompt with fixed 16-token chosen and rejected
continuations), epochs, learning rate, batch size, gradient accumulation, save / log cadence, and a
``metrics.json`` in the output directory. Local JSONL files take the place of hub dataset names (no
network). ``--use-lora`` trains low-rank adapters on the frozen model (``models/lora.py``) and saves the
merged model plus the adapters.

Both run on ``TrainEngine`` with per-row loss weights (``loss_weights=True``); the engine's fused
LM-head / cross-entropy kernel scales each row's gradient by its weight, so neither needs a kernel of
its own:

* SFT: weight 1/n on every row whose target token belongs to an assistant turn (n = such rows in the
  whole step, over all micro-batches), 0 on prompt, template and padding rows. The engine's loss is the
  mean cross-entropy over response tokens.
* DPO (Rafailov et al., 2023): L = mean_i -log sigmoid(z_i), z_i = beta * ((lp_c - lpref_c) -
  (lp_r - lpref_r)), lp = sum of the response tokens' log-probabilities = -sum_t ce_t. Its gradient is
  (beta / n) * sum_i sigmoid(-z_i) * (sum_{t in chosen_i} dce_t - sum_{t in rejected_i} dce_t): one
  weighted cross-entropy backward with weights +-beta * sigmoid(-z_i) / n on the two responses' rows is
  the exact DPO gradient. z_i comes from a forward-only pass at the same parameters
  (``TrainEngine.forward_loss``), the reference log-probabilities from one forward-only pass over the
  data with the initial weights (the frozen reference model).
"""
from __future__ import annotations

import json
import math
import os
import time
from dataclasses import asdict, dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

TEMPLATES = ("chatml", "llama", "zephyr")


# ───────────────────────────── tokenizers ─────────────────────────────
class ByteTokenizer:
    """UTF-8 bytes as token ids 3..258 (0 = pad, 1 = bos, 2 = eos): a tokenizer that needs no vocabulary
    file, for synthetic runs and tests (model vocabularies of at least 259)."""
    pad_id, bos_id, eos_id = 0, 1, 2
    vocab_size = 259

    def encode(self, text: str) -> List[int]:
        return [3 + b for b in text.encode("utf-8")]

    def decode(self, ids: Sequence[int]) -> str:
        return bytes(i - 3 for i in ids if 3 <= i < 259).decode("utf-8", "replace")


class FileTokenizer:
    """A ``tokenizers`` JSON tokenizer; pad / bos / eos are looked up among the usual special tokens."""

    def __init__(self, path: str):
        from tokenizers import Tokenizer
        self.tok = Tokenizer.from_file(path)
        self.vocab_size = self.tok.get_vocab_size()
        self.eos_id = self._first(("</s>", "<|endoftext|>", "<|im_end|>", "<eos>"), 0)
        self.pad_id = self._first(("<pad>", "<|pad|>"), self.eos_id)
        self.bos_id = self._first(("<s>", "<|begin_of_text|>", "<bos>"), self.eos_id)

    def _first(self, names, default: int) -> int:
        for n in names:
            i = self.tok.token_to_id(n)
            if i is not None:
                return int(i)
        return default

    def encode(self, text: str) -> List[int]:
        return self.tok.encode(text, add_special_tokens=False).ids

    def decode(self, ids: Sequence[int]) -> str:
        return self.tok.decode(list(ids))


# ───────────────────────────── chat data ─────────────────────────────
@dataclass
class Message:
    role: str  # "system" | "user" | "assistant"
    content: str


def render_chat(messages: Sequence[Message], template: str) -> List[Tuple[str, bool]]:
    """A conversation as text segments (text, trained): the assistant turns' content and their end
    marker are trained, everything else is context.

    chatml: ``<|im_start|>{role}\\n{content}<|im_end|>\\n`` per turn; zephyr: ``<|{role}|>\\n{content}</s>\\n``;
    llama (Llama-2 chat): ``<s>[INST] <<SYS>>\\n{system}\\n<</SYS>>\\n\\n{user} [/INST] {assistant} </s>``, the
    system prompt folded into the first user turn."""
    if template not in TEMPLATES:
        raise ValueError(f"unknown chat template {template!r} (one of {', '.join(TEMPLATES)})")
    segs: List[Tuple[str, bool]] = []
    if template in ("chatml", "zephyr"):
        for m in messages:
            if template == "chatml":
                head, end = f"<|im_start|>{m.role}\n", "<|im_end|>\n"
            else:
                head, end = f"<|{m.role}|>\n", "</s>\n"
            if m.role == "assistant":
                segs += [(head, False), (m.content + end, True)]
            else:
                segs.append((head + m.content + end, False))
        return segs
    system = ""
    for m in messages:
        if m.role == "system":
            system = m.content
        elif m.role == "user":
            u = m.content
            if system:
                u, system = f"<<SYS>>\n{system}\n<</SYS>>\n\n{u}", ""
            segs.append((f"<s>[INST] {u} [/INST]", False))
        else:
            segs.append((f" {m.content} </s>", True))
    return segs


@dataclass
class ChatExample:
    ids: List[int]
    trained: List[bool]  # per token: part of an assistant turn (a target of the loss)


def tokenize_conversation(messages: Sequence[Message], tok, template: str = "chatml",
                          max_seq_len: int = 512) -> ChatExample:
    """Each rendered segment is tokenized on its own, so a token never straddles a trained / context
    boundary; the example is cut to ``max_seq_len`` tokens."""
    ids: List[int] = []
    trained: List[bool] = []
    for text, tr in render_chat(messages, template):
        t = tok.encode(text)
        ids += t
        trained += [tr] * len(t)
    return ChatExample(ids[:max_seq_len], trained[:max_seq_len])


def synthetic_conversations(num_examples: int = 100) -> List[List[Message]]:
    """Five question / answer conversations behind a fixed system prompt, repeated (``run_sft.py:52-83``)."""
    qa = [("What is machine learning?", "Machine learning is a subset of artificial intelligence."),
          ("Tell me about Python.", "Python is a versatile programming language."),
          ("How far is the Earth from the Sun?",
           "The Earth orbits the Sun at a distance of about 93 million miles."),
          ("At what temperature does water boil?", "Water boils at 100 degrees Celsius at sea level."),
          ("What is photosynthesis?", "Photosynthesis converts sunlight into chemical energy in plants.")]
    out = []
    for i in range(num_examples):
        q, a = qa[i % len(qa)]
        out.append([Message("system", "You are a helpful assistant."), Message("user", q),
                    Message("assistant", a)])
    return out


_ROLES = {"system": "system", "user": "user", "human": "user", "assistant": "assistant", "gpt": "assistant"}


def _messages(turns) -> List[Message]:
    """Turns as ``{"role", "content"}`` or ShareGPT-style ``{"from": "system" | "human" | "gpt", "value"}``."""
    out = []
    for m in turns:
        role = m.get("role", m.get("from"))
        if role not in _ROLES:
            raise ValueError(f"unknown role {role!r}")
        out.append(Message(_ROLES[role], m.get("content", m.get("value"))))
    return out


def load_chat_jsonl(paths: Sequence[str], max_examples: Optional[int] = None) -> List[List[Message]]:
    """Conversations from JSONL files, one per line: ``{"messages": [{"role", "content"}, ...]}``,
    ShareGPT-style ``{"conversations": [{"from": "system" | "human" | "gpt", "value"}, ...]}`` (the
    layout of OpenHermes-2.5 and SlimOrca dumps) or ``{"prompt": ..., "response": ...}`` (also
    ``instruction`` / ``output``), at most ``max_examples`` per file."""
    out: List[List[Message]] = []
    for p in paths:
        n = 0
        with open(p) as f:
            for line in f:
                if not line.strip():
                    continue
                r = json.loads(line)
                if "messages" in r or "conversations" in r:
                    conv = _messages(r.get("messages", r.get("conversations")))
                else:
                    prompt = r.get("prompt", r.get("instruction"))
                    resp = r.get("response", r.get("output"))
                    if prompt is None or resp is None:
                        raise ValueError(f"{p}: a line needs 'messages' or a prompt / response pair")
                    conv = [Message("user", prompt), Message("assistant", resp)]
                out.append(conv)
                n += 1
                if max_examples is not None and n >= max_examples:
                    break
    return out


# ───────────────────────────── preference data ─────────────────────────────
@dataclass
class PreferencePair:
    """Token ids of the prompt and of the two full sequences (prompt + response), the convention of
    ``run_dpo.py:36-43``."""
    prompt_ids: List[int]
    chosen_ids: List[int]
    rejected_ids: List[int]


def synthetic_preferences(num_examples: int = 50) -> List[PreferencePair]:
    """Prompt 1..16, chosen continuation 17..32, rejected 33..48 (``run_dpo.py:40-55``)."""
    prompt = list(range(1, 17))
    return [PreferencePair(prompt, prompt + list(range(17, 33)), prompt + list(range(33, 49)))
            for _ in range(num_examples)]


def _preference_turns(r: dict) -> Tuple[List[Message], str, str]:
    """(context turns, chosen response, rejected response) of one preference line."""
    ch, rj = r["chosen"], r["rejected"]
    if isinstance(ch, list):  # whole conversations ending in the two assistant answers
        cm, rm = _messages(ch), _messages(rj)
        if not cm or cm[-1].role != "assistant" or not rm or rm[-1].role != "assistant":
            raise ValueError("chosen / rejected conversations must end with an assistant turn")
        return cm[:-1], cm[-1].content, rm[-1].content
    prompt = r["prompt"]
    context = _messages(prompt) if isinstance(prompt, list) else [Message("user", prompt)]
    return context, ch, rj


def _preference_ids(context: List[Message], resp: str, tok, template: str) -> Tuple[List[int], List[int]]:
    """(prompt ids: everything the template renders before the final answer, answer ids)."""
    segs = render_chat(list(context) + [Message("assistant", resp)], template)
    last = max(i for i, (_, tr) in enumerate(segs) if tr)
    return sum((tok.encode(t) for t, _ in segs[:last]), []), tok.encode(segs[last][0])


def load_preference_jsonl(paths: Sequence[str], tok, template: str = "chatml",
                          max_examples: Optional[int] = None) -> List[PreferencePair]:
    """Pairs from JSONL lines ``{"prompt": str | [turns], "chosen": str, "rejected": str}`` (the prompt
    as the context turns of the chat template, each response as the assistant turn that follows) or
    ``{"chosen": [turns], "rejected": [turns]}`` whose two conversations share all but their last,
    assistant, turn (the layout of binarized preference sets)."""
    out: List[PreferencePair] = []
    for p in paths:
        n = 0
        with open(p) as f:
            for line in f:
                if not line.strip():
                    continue
                context, chosen, rejected = _preference_turns(json.loads(line))
                prompt, c_ids = _preference_ids(context, chosen, tok, template)
                _, r_ids = _preference_ids(context, rejected, tok, template)
                out.append(PreferencePair(prompt, prompt + c_ids, prompt + r_ids))
                n += 1
                if max_examples is not None and n >= max_examples:
                    break
    return out


# ───────────────────────────── batches and loss weights ─────────────────────────────
def pack_rows(seqs: Sequence[Sequence[int]], trained: Sequence[Sequence[bool]], seq_len: int,
              pad_id: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Sequences -> ids [n, seq_len] int32 (cut / padded with ``pad_id``) and the loss mask [n, seq_len-1]:
    row t (predicting token t+1) is 1 when token t+1 exists and is trained."""
    n = len(seqs)
    ids = torch.full((n, seq_len), pad_id, dtype=torch.int32)
    mask = torch.zeros(n, seq_len - 1, dtype=torch.float32)
    for i, (s, tr) in enumerate(zip(seqs, trained)):
        s, tr = list(s)[:seq_len], list(tr)[:seq_len]
        if s:
            ids[i, :len(s)] = torch.tensor(s, dtype=torch.int32)
        if len(s) > 1:
            mask[i, :len(s) - 1] = torch.tensor(tr[1:], dtype=torch.float32)
    return ids, mask


def sft_weights(mask: torch.Tensor) -> torch.Tensor:
    """Loss weights of one SFT step: the mask divided by its count (the mean over trained rows)."""
    return mask / max(float(mask.sum()), 1.0)


def pair_rows(pairs: Sequence[PreferencePair], seq_len: int, pad_id: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Pairs -> ids [2n, seq_len] with chosen sequence i at row 2i and rejected at 2i+1, and the mask of
    response rows (targets at positions >= len(prompt))."""
    seqs, trained = [], []
    for p in pairs:
        for s in (p.chosen_ids, p.rejected_ids):
            seqs.append(s)
            trained.append([j >= len(p.prompt_ids) for j in range(len(s))])
    return pack_rows(seqs, trained, seq_len, pad_id)


def sequence_logps(row_ce: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """Sum of the masked rows' log-probabilities per sequence: -sum_t ce[., t] * mask[., t]."""
    return -(row_ce.double() * mask.double()).sum(-1)


def dpo_weights(lp: torch.Tensor, ref_lp: torch.Tensor, mask: torch.Tensor, beta: float
                ) -> Tuple[torch.Tensor, Dict[str, float]]:
    """Loss weights whose weighted cross-entropy gradient is the DPO gradient, and the step's statistics.

    ``lp`` / ``ref_lp``: [2n] sequence log-probabilities of the policy and the reference (chosen at even,
    rejected at odd rows); ``mask``: [2n, T] response rows."""
    lp, ref_lp = lp.double(), ref_lp.double()
    r = beta * (lp - ref_lp)
    rc, rr = r[0::2], r[1::2]
    z = rc - rr
    n = z.numel()
    coef = beta * torch.sigmoid(-z) / n
    sign = torch.ones(2 * n, dtype=torch.float64)
    sign[1::2] = -1.0
    w = (mask.double() * (coef.repeat_interleave(2) * sign)[:, None]).float()
    stats = {"loss": float(torch.nn.functional.softplus(-z).mean()),
             "reward_accuracy": float((z > 0).double().mean()),
             "reward_margin": float(z.mean()),
             "chosen_reward": float(rc.mean()),
             "rejected_reward": float(rr.mean())}
    return w, stats


# ───────────────────────────── trainers ─────────────────────────────
@dataclass
class SFTConfig:
    learning_rate: float = 2e-5
    num_epochs: int = 3
    batch_size: int = 4  # sequences per micro-batch
    gradient_accumulation_steps: int = 8
    max_seq_len: int = 512
    warmup_fraction: float = 0.03
    min_lr_fraction: float = 0.1  # cosine decay to this fraction of the learning rate
    weight_decay: float = 0.0
    grad_clip_norm: float = 1.0
    save_every_n_steps: int = 500
    log_every_n_steps: int = 10
    output_dir: str = "models/sft"
    seed: int = 0
    cuda_graph: bool = True  # replay each step as one captured CUDA graph (full fine-tuning)
    use_lora: bool = False  # train rank-r adapters on the frozen weights instead
    lora_rank: int = 64
    lora_alpha: float = 128.0


@dataclass
class DPOConfig:
    beta: float = 0.1
    learning_rate: float = 5e-7
    num_epochs: int = 1
    batch_size: int = 2  # preference pairs per micro-batch (two sequences each)
    gradient_accumulation_steps: int = 16
    max_seq_len: int = 256
    warmup_fraction: float = 0.1
    min_lr_fraction: float = 0.1
    weight_decay: float = 0.0
    grad_clip_norm: float = 1.0
    save_every_n_steps: int = 200
    log_every_n_steps: int = 10
    output_dir: str = "models/dpo"
    seed: int = 0
    cuda_graph: bool = True
    use_lora: bool = False
    lora_rank: int = 64
    lora_alpha: float = 128.0


def step_order(n_items: int, per_step: int, epochs: int, seed: int) -> List[List[int]]:
    """Item indices of every step: a fresh permutation per epoch, cut into steps of ``per_step``; the last
    step of an epoch is filled from the start of the same permutation."""
    if n_items <= 0:
        raise ValueError("no training examples")
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(epochs):
        perm = torch.randperm(n_items, generator=g).tolist()
        for s in range(max(1, math.ceil(n_items / per_step))):
            out.append([perm[(s * per_step + j) % n_items] for j in range(per_step)])
    return out


class OracleEngine:
    """The subset of ``TrainEngine`` the trainers use, on the CPU: the fp32 PyTorch formulation of the
    model (``models/oracle.py``) with autograd and the reference optimiser's AdamW (per-tensor
    clipping), the same per-row loss weights and the same forward-only per-row losses. The reference's
    post-training scripts default to the CPU for their synthetic smoke runs; this keeps ``sft`` / ``dpo``
    usable there (slowly)."""

    def __init__(self, cfg, batch: int, seq_len: int, optim, flat_init: torch.Tensor, grad_accum: int = 1,
                 loss_weights: bool = True):
        from .models.oracle import AdamWRef
        from .models.params import ParamLayout
        self.cfg, self.B, self.S, self.A, self.T = cfg, batch, seq_len, max(int(grad_accum), 1), seq_len - 1
        self.device = torch.device("cpu")
        self.params = {k: v.detach().clone().float().requires_grad_() for k, v in
                       ParamLayout(cfg).views(flat_init).items()}
        self.opt = AdamWRef(self.params, lr=optim.lr, betas=(optim.beta1, optim.beta2), eps=optim.eps,
                            weight_decay=optim.weight_decay, clip=optim.grad_clip_norm,
                            clip_global=optim.clip_global)
        self.lr = optim.lr
        self.ids = torch.zeros(self.A * batch, seq_len, dtype=torch.int32)
        self.loss_w = torch.zeros(self.A * batch * self.T) if loss_weights else None
        self.loss = torch.zeros(4)
        self.graph = None

    def set_tokens(self, tokens: torch.Tensor):
        self.ids.copy_(tokens)

    def set_loss_weights(self, w: torch.Tensor):
        self.loss_w.copy_(w.reshape(-1).float())

    def set_lr(self, lr: float):
        self.lr = lr

    def _row_ce(self, micro: int) -> torch.Tensor:
        from .models import oracle
        ids = self.ids[micro * self.B:(micro + 1) * self.B].long()
        z = oracle.logits_fn(self.params, self.cfg, ids[:, :-1], mask_value=None)
        return -torch.log_softmax(z.float(), dim=-1).gather(-1, ids[:, 1:, None])[..., 0]

    def forward_loss(self, micro: int = 0) -> torch.Tensor:
        with torch.no_grad():
            return self._row_ce(micro).reshape(-1)

    def step(self):
        n = self.B * self.T
        total = 0.0
        for a in range(self.A):
            w = (self.loss_w[a * n:(a + 1) * n].view(self.B, self.T) if self.loss_w is not None
                 else torch.full((self.B, self.T), 1.0 / (n * self.A)))
            ce = self._row_ce(a)
            l = (w * torch.where(w != 0, ce, torch.zeros_like(ce))).sum()
            l.backward()
            total += float(l.detach())
        finite = math.isfinite(total)
        self.loss[0], self.loss[1] = total, 0.0 if finite else 1.0
        if finite:
            self.opt.step(self.lr)
        else:  # skipped like a non-finite step on the GPU
            for q in self.params.values():
                q.grad = None

    def state_dict(self) -> Dict[str, torch.Tensor]:
        return {k: v.detach().float().cpu().clone() for k, v in self.params.items()}


class _EngineTrainer:
    """What both trainers share: a TrainEngine with per-row loss weights (``OracleEngine`` on the CPU),
    the learning-rate schedule, checkpoints and the metrics file."""

    def __init__(self, model_cfg, flat: torch.Tensor, batch: int, c, device: str):
        from .config import OptimConfig
        from .models.engine import TrainEngine
        if c.max_seq_len > model_cfg.max_seq_len:
            model_cfg.max_seq_len = c.max_seq_len
        self.cfg, self.c, self.B, self.A = model_cfg, c, batch, c.gradient_accumulation_steps
        self.S = c.max_seq_len
        optim = OptimConfig(lr=c.learning_rate, weight_decay=c.weight_decay, grad_clip_norm=c.grad_clip_norm)
        if torch.device(device).type == "cpu":
            if c.use_lora:
                raise ValueError("LoRA adapters train on the CUDA engine: use a cuda device")
            self.eng = OracleEngine(model_cfg, batch, self.S, optim, flat, grad_accum=self.A)
        else:
            self.eng = TrainEngine(model_cfg, batch, self.S, device=device, flat_init=flat, grad_accum=self.A,
                                   optim=optim, loss_weights=True)
        self.dev = self.eng.device
        self.lora = None
        if c.use_lora:
            from .models.lora import LoraAdapters
            self.lora = LoraAdapters(self.eng, c.lora_rank, c.lora_alpha, lr=c.learning_rate,
                                     weight_decay=c.weight_decay, grad_clip_norm=c.grad_clip_norm, seed=c.seed)
        self.history: List[dict] = []
        os.makedirs(c.output_dir, exist_ok=True)

    def _lr(self, k: int, total: int) -> float:
        from .config import cosine_lr
        c = self.c
        return cosine_lr(k, int(total * c.warmup_fraction), total, c.learning_rate,
                         c.learning_rate * c.min_lr_fraction)

    def _run_step(self, k: int, total: int, weights: torch.Tensor):
        self.eng.set_loss_weights(weights.to(self.dev))
        if self.lora is not None:
            self.lora.set_lr(self._lr(k, total))
            self.lora.step()
            return
        self.eng.set_lr(self._lr(k, total))
        if k == 0 and self.c.cuda_graph and self.dev.type == "cuda":
            self.eng.capture()
        self.eng.step()

    def _sync(self):
        if self.dev.type == "cuda":
            torch.cuda.synchronize(self.dev)

    def _want_log(self, k: int, total: int) -> bool:
        return k == 0 or k + 1 == total or (k + 1) % max(self.c.log_every_n_steps, 1) == 0

    def save(self, name: str) -> str:
        """The model (adapters folded in when training LoRA, whose adapters go to ``adapter_<name>``)."""
        from .utils.checkpoint import save_safetensors
        path = os.path.join(self.c.output_dir, name)
        if self.lora is not None:
            save_safetensors(self.lora.merged_state_dict(), path)
            save_safetensors(self.lora.adapter_state_dict(), os.path.join(self.c.output_dir, "adapter_" + name))
        else:
            save_safetensors(self.eng.state_dict(), path)
        return path

    def _finish(self, metrics: dict) -> dict:
        metrics["checkpoint"] = self.save("model.safetensors")
        if self.lora is not None:
            metrics["adapter"] = os.path.join(self.c.output_dir, "adapter_model.safetensors")
            metrics["trainable_params"] = self.lora.total
        metrics["config"] = asdict(self.c)
        with open(os.path.join(self.c.output_dir, "metrics.json"), "w") as f:
            json.dump(metrics, f, indent=2)
        return metrics


class SFTTrainer(_EngineTrainer):
    """Supervised fine-tuning with the loss on assistant tokens (mean over the step's response rows)."""

    def __init__(self, model_cfg, flat: torch.Tensor, examples: Sequence[ChatExample], config: SFTConfig,
                 pad_id: int = 0, device: str = "cuda:0"):
        super().__init__(model_cfg, flat, config.batch_size, config, device)
        self.examples, self.pad_id = list(examples), pad_id

    def train(self, log=print) -> dict:
        c = self.c
        order = step_order(len(self.examples), self.B * self.A, c.num_epochs, c.seed)
        total, resp = len(order), 0
        t0 = time.perf_counter()
        for k, idx in enumerate(order):
            ex = [self.examples[i] for i in idx]
            ids, mask = pack_rows([e.ids for e in ex], [e.trained for e in ex], self.S, self.pad_id)
            self.eng.set_tokens(ids.to(self.dev))
            self._run_step(k, total, sft_weights(mask))
            resp += int(mask.sum())
            if self._want_log(k, total):
                rec = {"step": k + 1, "loss": float(self.eng.loss[0]), "lr": self._lr(k, total)}
                self.history.append(rec)
                log(json.dumps({"event": "sft", **rec}))
            if c.save_every_n_steps and (k + 1) % c.save_every_n_steps == 0:
                self.save(f"step_{k + 1}.safetensors")
        self._sync()
        dt = time.perf_counter() - t0
        return self._finish({"steps": total, "epochs": c.num_epochs, "examples": len(self.examples),
                             "response_tokens": resp, "tokens_per_sec": total * self.B * self.A * self.S / dt,
                             "first_loss": self.history[0]["loss"], "final_loss": self.history[-1]["loss"],
                             "history": self.history})


class DPOTrainer(_EngineTrainer):
    """Direct preference optimisation against the frozen initial model (the reference policy)."""

    def __init__(self, model_cfg, flat: torch.Tensor, pairs: Sequence[PreferencePair], config: DPOConfig,
                 pad_id: int = 0, device: str = "cuda:0"):
        super().__init__(model_cfg, flat, 2 * config.batch_size, config, device)
        self.pairs, self.pad_id = list(pairs), pad_id
        self.per_step = config.batch_size * self.A

    def _logps(self, mask: torch.Tensor) -> torch.Tensor:
        """Sequence log-probabilities of the step's sequences at the current weights (forward only)."""
        m = mask.to(self.dev)
        T = self.S - 1
        out = []
        for a in range(self.A):
            rows = self.eng.forward_loss(a).view(self.B, T)
            out.append(sequence_logps(rows, m[a * self.B:(a + 1) * self.B]))
        return torch.cat(out).cpu()

    def reference_logps(self) -> torch.Tensor:
        """[n_pairs, 2] (chosen, rejected) log-probabilities under the initial weights."""
        n = len(self.pairs)
        ref = torch.zeros(n, 2, dtype=torch.float64)
        for s in range(0, n, self.per_step):
            idx = [(s + j) % n for j in range(self.per_step)]
            ids, mask = pair_rows([self.pairs[i] for i in idx], self.S, self.pad_id)
            self.eng.set_tokens(ids.to(self.dev))
            lp = self._logps(mask).view(-1, 2)
            for j, i in enumerate(idx):
                ref[i] = lp[j]
        return ref

    def train(self, log=print) -> dict:
        c = self.c
        ref = self.reference_logps()
        order = step_order(len(self.pairs), self.per_step, c.num_epochs, c.seed)
        total = len(order)
        t0 = time.perf_counter()
        for k, idx in enumerate(order):
            ids, mask = pair_rows([self.pairs[i] for i in idx], self.S, self.pad_id)
            self.eng.set_tokens(ids.to(self.dev))
            lp = self._logps(mask)
            w, st = dpo_weights(lp, ref[idx].reshape(-1), mask, c.beta)
            self._run_step(k, total, w)
            if self._want_log(k, total):
                rec = {"step": k + 1, **st, "lr": self._lr(k, total)}
                self.history.append(rec)
                log(json.dumps({"event": "dpo", **rec}))
            if c.save_every_n_steps and (k + 1) % c.save_every_n_steps == 0:
                self.save(f"step_{k + 1}.safetensors")
        self._sync()
        dt = time.perf_counter() - t0
        return self._finish({"steps": total, "epochs": c.num_epochs, "pairs": len(self.pairs),
                             "pairs_per_sec": total * self.per_step / dt,
                             "first_loss": self.history[0]["loss"], "final_loss": self.history[-1]["loss"],
                             "final_reward_accuracy": self.history[-1]["reward_accuracy"],
                             "history": self.history})
