"""Text generation from a checkpoint: the sampler behind ``cli.py generate`` and an OpenAI-style
completion server (``cli.py serve``) on the native HTTP server.

The reference's node samples by re-running the full forward for every new token (no KV cache,
``node/cli/src/main.rs:1416-1548``); its serving script (``scripts/serve.py:16,32-37``) exposes an
OpenAI-style API but imports a package that is not in its repository. Here both re-run the forward
per token as well: on a GPU through the CUDA engine (``EngineLM``: a forward-only engine over a fixed
window, the logits of the last real position from its final hidden row and the tied embedding; causal
attention makes the padding after that position irrelevant), on the CPU through the model's plain
PyTorch formulation (``models/oracle.py``).

Routes: ``POST /v1/completions`` with {"prompt": text or [token ids], "max_tokens", "temperature",
"seed", "stop_token"} -> {"id", "object": "text_completion", "created", "model", "choices": [{"text",
"token_ids", "index", "finish_reason"}], "usage": {"prompt_tokens", "completion_tokens",
"total_tokens"}}; ``POST /v1/chat/completions`` with {"messages": [{"role", "content"}], "max_tokens",
"temperature", "seed", "template"} -> {"object": "chat.completion", "choices": [{"message": {"role":
"assistant", "content"}, "finish_reason"}], "usage"}: the conversation is rendered with the chat
template the model was fine-tuned with (chatml by default) and generation stops at the template's end
marker; ``GET /v1/models``; ``GET /health``. Text needs a tokenizer (a file, or ``bytes`` for the UTF-8
byte tokenizer of the post-training commands).
"""
from __future__ import annotations

import ctypes
import json
import threading
import time
import uuid
from typing import Callable, List, Optional, Tuple

import torch


class EngineLM:
    """Next-token logits from the CUDA forward of forward-only engines (one sequence each). Each context
    runs on the smallest of the power-of-two windows (128 .. ``window`` input positions) that holds it,
    so a token costs a forward over about its context, not over the longest one; the engines are made on
    first use and share one copy of the weights. Longer contexts keep their last ``window`` tokens."""

    MIN_WINDOW = 128

    def __init__(self, sd, cfg, device: str = "cuda:0", window: int = 1024):
        from .models.engine import TrainEngine
        from .models.params import ParamLayout
        L = ParamLayout(cfg)
        flat = torch.zeros(L.total)
        L.load_state_dict(flat, {k: v.detach().float().cpu() for k, v in sd.items()})
        cfg.max_seq_len = max(cfg.max_seq_len, window + 1)
        self.cfg, self.device, self.window = cfg, device, int(window)
        self.windows = self.window_sizes(self.window)
        # the largest engine holds the weights; the others are made when a context first fits them
        self.engines = {self.window: TrainEngine(cfg, 1, self.window + 1, device=device, flat_init=flat,
                                                 inference=True)}
        self.eng = self.engines[self.window]

    @classmethod
    def window_sizes(cls, window: int) -> List[int]:
        """Powers of two from MIN_WINDOW below ``window``, then ``window`` itself."""
        out, w = [], min(cls.MIN_WINDOW, window)
        while w < window:
            out.append(w)
            w *= 2
        return out + [window]

    def _engine(self, n: int):
        w = next(w for w in self.windows if w >= n)
        if w not in self.engines:
            from .models.engine import TrainEngine
            self.engines[w] = TrainEngine(self.cfg, 1, w + 1, device=self.device, inference=True,
                                          weights_from=self.eng)
        return self.engines[w]

    def next_logits(self, seq: List[int]) -> torch.Tensor:
        """fp32 logits (CPU) of the token after ``seq``."""
        ctx = seq[-self.window:]
        eng = self._engine(len(ctx))
        row = torch.zeros(1, eng.S, dtype=torch.int32)
        row[0, :len(ctx)] = torch.tensor(ctx, dtype=torch.int32)
        eng.set_tokens(row.to(eng.device))
        xs = eng.forward_hidden(0)
        with torch.no_grad():
            return (xs[len(ctx) - 1:len(ctx)].float() @ eng.E.t())[0].cpu()


def sample(sd, cfg, ids: List[int], max_tokens: int, temperature: float = 0.0, seed: int = 0,
           stop_token: Optional[int] = None, lm: Optional[EngineLM] = None,
           stop_fn: Optional[Callable[[List[int]], bool]] = None) -> Tuple[List[int], str]:
    """Appends up to ``max_tokens`` tokens to ``ids`` (greedy at temperature <= 0, else softmax sampling
    from a generator seeded with ``seed``); returns the new tokens and the finish reason ("length" or
    "stop": ``stop_token`` sampled, or ``stop_fn(new tokens)`` true). With ``lm`` the logits come from
    the CUDA engine, else from the PyTorch formulation."""
    from .models import oracle
    dev = next(iter(sd.values())).device
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    seq = list(ids) if ids else [1]
    out: List[int] = []
    with torch.no_grad():
        for _ in range(int(max_tokens)):
            if lm is not None:
                z = lm.next_logits(seq)
            else:
                x = torch.tensor([seq[-cfg.max_seq_len:]], device=dev)
                z = oracle.logits_fn(sd, cfg, x)[0, -1].float().cpu()
            if temperature <= 0:
                nxt = int(z.argmax())
            else:
                nxt = int(torch.multinomial(torch.softmax(z / temperature, -1), 1, generator=g))
            seq.append(nxt)
            out.append(nxt)
            if (stop_token is not None and nxt == stop_token) or (stop_fn is not None and stop_fn(out)):
                return out, "stop"
    return out, "length"


def load_model(checkpoint: str, device: str = "cpu", rope_theta: Optional[float] = None, min_len: int = 0):
    """Checkpoint (safetensors) -> (weights on ``device``, ModelConfig inferred from the shapes)."""
    from .cli import _infer_model_config
    from .utils.checkpoint import load_safetensors
    sd = load_safetensors(checkpoint)
    cfg = _infer_model_config(sd)
    if rope_theta:
        cfg.rope_theta = rope_theta
    cfg.max_seq_len = max(cfg.max_seq_len, min_len)
    sd = {k: v.to(device) for k, v in sd.items()}
    return sd, cfg


class CompletionServer:
    """OpenAI-style completions for one checkpoint; requests are served one at a time (the model's
    forward is not re-entrant on one device)."""

    def __init__(self, checkpoint: str, device: str = "cpu", tokenizer: Optional[str] = None,
                 rope_theta: Optional[float] = None, model_name: Optional[str] = None, max_tokens_cap: int = 1024,
                 template: str = "chatml"):
        import os
        if os.path.isdir(checkpoint):  # a model directory, as the reference's serve script takes
            checkpoint = os.path.join(checkpoint, "model.safetensors")
        self.sd, self.cfg = load_model(checkpoint, device, rope_theta, min_len=max_tokens_cap + 64)
        self.template = template
        # on a GPU the forward runs on the CUDA engine; its window covers the longest request
        self.lm = (EngineLM(self.sd, self.cfg, device, window=self.cfg.max_seq_len)
                   if torch.device(device).type == "cuda" else None)
        self.tok = None
        if tokenizer == "bytes":
            from .alignment import ByteTokenizer
            self.tok = ByteTokenizer()
        elif tokenizer:
            from .alignment import FileTokenizer
            self.tok = FileTokenizer(tokenizer)
        self.model = model_name or checkpoint.rsplit("/", 1)[-1]
        self.cap = max_tokens_cap
        self._lock = threading.Lock()
        self.handle = None
        self.port = None

    # ── request handling (pure: testable without sockets) ──
    def complete(self, req: dict) -> Tuple[int, dict]:
        prompt = req.get("prompt", "")
        if isinstance(prompt, list) and len(prompt) == 1 and isinstance(prompt[0], (str, list)):
            prompt = prompt[0]
        if isinstance(prompt, list):
            ids = [int(t) for t in prompt]
        elif self.tok is not None:
            # plain prompts are tokenized like the pretraining shards (with the tokenizer's own special
            # tokens, e.g. a leading BOS); chat prompts like the fine-tuning commands (without)
            raw = getattr(self.tok, "tok", None)
            ids = raw.encode(str(prompt)).ids if raw is not None else self.tok.encode(str(prompt))
        else:
            return 400, {"error": {"message": "text prompts need a tokenizer (start with --tokenizer) or a list "
                                              "of token ids", "type": "invalid_request_error"}}
        n = int(req.get("max_tokens", 16))
        if n < 0 or n > self.cap:
            return 400, {"error": {"message": f"max_tokens must be in [0, {self.cap}]",
                                   "type": "invalid_request_error"}}
        bad = [t for t in ids if t < 0 or t >= self.cfg.vocab_size]
        if bad:
            return 400, {"error": {"message": f"token id {bad[0]} outside the vocabulary",
                                   "type": "invalid_request_error"}}
        stop = req.get("stop_token")
        with self._lock:
            new, reason = sample(self.sd, self.cfg, ids, n, float(req.get("temperature", 0.0)),
                                 int(req.get("seed", 0)), int(stop) if stop is not None else None, lm=self.lm)
        text = self.tok.decode(new) if self.tok is not None else None
        return 200, {"id": f"cmpl-{uuid.uuid4().hex[:24]}", "object": "text_completion", "created": int(time.time()),
                     "model": self.model,
                     "choices": [{"text": text, "token_ids": new, "index": 0, "finish_reason": reason}],
                     "usage": {"prompt_tokens": len(ids), "completion_tokens": len(new),
                               "total_tokens": len(ids) + len(new)}}

    def chat(self, req: dict) -> Tuple[int, dict]:
        """Chat completion: the messages rendered with the chat template, the answer generated up to the
        template's end marker (or max_tokens)."""
        from .alignment import Message, render_chat
        bad = lambda msg: (400, {"error": {"message": msg, "type": "invalid_request_error"}})
        if self.tok is None:
            return bad("chat needs a tokenizer (start with --tokenizer FILE, or --tokenizer bytes)")
        msgs = req.get("messages")
        if not isinstance(msgs, list) or not msgs or not all(
                isinstance(m, dict) and m.get("role") in ("system", "user", "assistant") and
                isinstance(m.get("content"), str) for m in msgs):
            return bad("messages must be a non-empty list of {role: system | user | assistant, content}")
        try:
            segs = render_chat([Message(m["role"], m["content"]) for m in msgs] + [Message("assistant", "")],
                               req.get("template", self.template))
        except ValueError as e:
            return bad(str(e))
        end = segs[-1][0].strip()  # what the template appends to an (empty) answer: its end marker
        ids = self.tok.encode("".join(t for t, _ in segs[:-1]))
        n = int(req.get("max_tokens", 64))
        if n < 0 or n > self.cap:
            return bad(f"max_tokens must be in [0, {self.cap}]")
        if any(t >= self.cfg.vocab_size for t in ids):
            return bad("the tokenizer's ids do not fit the model's vocabulary")
        with self._lock:
            new, reason = sample(self.sd, self.cfg, ids, n, float(req.get("temperature", 0.0)),
                                 int(req.get("seed", 0)), lm=self.lm,
                                 stop_fn=lambda out: end in self.tok.decode(out[-64:]))
        text = self.tok.decode(new)
        if end in text:
            text, reason = text[:text.index(end)], "stop"
        return 200, {"id": f"chatcmpl-{uuid.uuid4().hex[:24]}", "object": "chat.completion",
                     "created": int(time.time()), "model": self.model,
                     "choices": [{"index": 0, "message": {"role": "assistant", "content": text.strip()},
                                  "finish_reason": reason}],
                     "usage": {"prompt_tokens": len(ids), "completion_tokens": len(new),
                               "total_tokens": len(ids) + len(new)}}

    def handle_request(self, method: str, path: str, body: bytes) -> Tuple[int, dict]:
        route = path.split("?", 1)[0]
        if method == "GET" and route == "/health":
            return 200, {"status": "ok"}
        if method == "GET" and route == "/v1/models":
            return 200, {"object": "list", "data": [{"id": self.model, "object": "model", "owned_by": "distrain"}]}
        if method == "POST" and route in ("/v1/completions", "/v1/chat/completions"):
            try:
                req = json.loads(body or b"{}")
            except ValueError:
                return 400, {"error": {"message": "body is not JSON", "type": "invalid_request_error"}}
            return self.complete(req) if route == "/v1/completions" else self.chat(req)
        return 404, {"error": {"message": f"no route {method} {route}", "type": "not_found"}}

    # ── native HTTP server ──
    def start(self, host: str = "0.0.0.0", port: int = 8000, threads: int = 4) -> int:
        from .utils import native
        handler_t = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_void_p,
                                     ctypes.c_longlong, ctypes.c_void_p)
        L = native.rt()
        native.register("dtr_http_start", [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, handler_t,
                                           ctypes.c_void_p], ctypes.c_void_p)
        native.register("dtr_http_port", [ctypes.c_void_p], ctypes.c_int)
        native.register("dtr_http_stop", [ctypes.c_void_p], None)
        native.register("dtr_http_respond", [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_void_p,
                                             ctypes.c_longlong], None)

        def on_request(ctx, method, path, body, blen, resp):
            try:
                data = ctypes.string_at(body, blen) if blen else b""
                status, obj = self.handle_request(method.decode(), path.decode(), data)
            except Exception as e:  # the server thread must answer whatever happens
                status, obj = 500, {"error": {"message": str(e), "type": "server_error"}}
            out = json.dumps(obj).encode()
            L.dtr_http_respond(resp, status, b"application/json", out, len(out))

        self._cb = handler_t(on_request)
        self.handle = L.dtr_http_start(host.encode(), port, threads, 1 << 20, self._cb, None)
        if not self.handle:
            raise RuntimeError(f"serve: cannot bind {host}:{port}")
        self.port = L.dtr_http_port(self.handle)
        return self.port

    def stop(self):
        if self.handle:
            from .utils import native
            native.rt().dtr_http_stop(self.handle)
            self.handle = None
