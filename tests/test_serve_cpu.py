"""OpenAI-style completion server on CPU: request validation, greedy output equal to the sampler (and to
``cli.py generate``), seeded sampling, and one round trip over the native HTTP server."""
import json
import urllib.request

import pytest
import torch


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from distrain_b200.config import preset
    from distrain_b200.models.params import ParamLayout, init_flat
    from distrain_b200.utils.checkpoint import save_safetensors
    cfg = preset("micro")
    L = ParamLayout(cfg)
    flat = init_flat(L, seed=3)
    path = str(tmp_path_factory.mktemp("ck") / "model.safetensors")
    save_safetensors(L.to_state_dict(flat), path)
    return path


def test_completions_validate_and_match_the_sampler(ckpt):
    from distrain_b200.serve import CompletionServer, sample
    srv = CompletionServer(ckpt, "cpu", max_tokens_cap=64)
    st, out = srv.handle_request("POST", "/v1/completions", json.dumps({"prompt": [1, 2, 3], "max_tokens": 6}).encode())
    assert st == 200, out
    ch = out["choices"][0]
    assert out["object"] == "text_completion" and ch["finish_reason"] == "length" and len(ch["token_ids"]) == 6
    assert out["usage"] == {"prompt_tokens": 3, "completion_tokens": 6, "total_tokens": 9}
    ref, _ = sample(srv.sd, srv.cfg, [1, 2, 3], 6)
    assert ch["token_ids"] == ref
    # seeded sampling is reproducible; a stop token ends the completion early
    body = {"prompt": [5, 6], "max_tokens": 8, "temperature": 1.0, "seed": 11}
    a = srv.handle_request("POST", "/v1/completions", json.dumps(body).encode())[1]["choices"][0]["token_ids"]
    b = srv.handle_request("POST", "/v1/completions", json.dumps(body).encode())[1]["choices"][0]["token_ids"]
    assert a == b
    body["stop_token"] = a[2]
    c = srv.handle_request("POST", "/v1/completions", json.dumps(body).encode())[1]["choices"][0]
    assert c["finish_reason"] == "stop" and c["token_ids"] == a[:a.index(a[2]) + 1]
    # invalid requests: text without a tokenizer, too many tokens, ids outside the vocabulary, bad JSON
    assert srv.handle_request("POST", "/v1/completions", b'{"prompt": "hi"}')[0] == 400
    assert srv.handle_request("POST", "/v1/completions", b'{"prompt": [1], "max_tokens": 65}')[0] == 400
    assert srv.handle_request("POST", "/v1/completions", json.dumps({"prompt": [srv.cfg.vocab_size]}).encode())[0] == 400
    assert srv.handle_request("POST", "/v1/completions", b"{not json")[0] == 400
    assert srv.handle_request("GET", "/nope", b"")[0] == 404
    models = srv.handle_request("GET", "/v1/models", b"")[1]
    assert models["data"][0]["id"] == srv.model


def test_server_round_trip(ckpt):
    from distrain_b200.serve import CompletionServer
    srv = CompletionServer(ckpt, "cpu", max_tokens_cap=16)
    port = srv.start("127.0.0.1", 0, threads=2)
    try:
        req = urllib.request.Request(f"http://127.0.0.1:{port}/v1/completions", method="POST",
                                     data=json.dumps({"prompt": [[1, 2]], "max_tokens": 3}).encode(),
                                     headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=60) as r:
            out = json.loads(r.read())
        assert len(out["choices"][0]["token_ids"]) == 3
        with urllib.request.urlopen(f"http://127.0.0.1:{port}/health", timeout=10) as r:
            assert json.loads(r.read())["status"] == "ok"
    finally:
        srv.stop()


def test_engine_window_ladder():
    """Forward windows of the GPU sampler: powers of two from 128 up to the longest context."""
    from distrain_b200.serve import EngineLM
    assert EngineLM.window_sizes(300) == [128, 256, 300]
    assert EngineLM.window_sizes(128) == [128]
    assert EngineLM.window_sizes(100) == [100]
    assert EngineLM.window_sizes(4096) == [128, 256, 512, 1024, 2048, 4096]


def test_chat_completions(tmp_path, monkeypatch):
    """/v1/chat/completions: the conversation goes through the chat template, the answer stops at the
    template's end marker, and the server takes a model directory and a model name."""
    from distrain_b200 import serve
    from distrain_b200.alignment import ByteTokenizer
    from distrain_b200.config import ModelConfig
    from distrain_b200.models.params import ParamLayout, init_flat
    from distrain_b200.utils.checkpoint import save_safetensors
    cfg = ModelConfig(hidden_dim=32, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=64, vocab_size=260,
                      max_seq_len=256, rope_theta=10000.0)
    L = ParamLayout(cfg)
    save_safetensors(L.to_state_dict(init_flat(L, seed=2)), str(tmp_path / "model.safetensors"))
    srv = serve.CompletionServer(str(tmp_path), "cpu", tokenizer="bytes", model_name="tiny-chat", max_tokens_cap=64)
    assert srv.model == "tiny-chat"
    body = {"messages": [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"}],
            "max_tokens": 5}
    st, out = srv.handle_request("POST", "/v1/chat/completions", json.dumps(body).encode())
    assert st == 200, out
    assert out["object"] == "chat.completion" and out["choices"][0]["message"]["role"] == "assistant"
    assert out["usage"]["completion_tokens"] == 5 and out["choices"][0]["finish_reason"] == "length"
    # the prompt is the chatml rendering up to the assistant header
    tok = ByteTokenizer()
    want = "<|im_start|>system\nbe brief<|im_end|>\n<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n"
    assert out["usage"]["prompt_tokens"] == len(tok.encode(want))
    # generation stops at the end marker, which is cut from the answer
    reply = tok.encode("Hello!<|im_end|>\nextra")

    def fake_sample(sd, cfg, ids, n, temperature=0.0, seed=0, stop_token=None, lm=None, stop_fn=None):
        assert tok.decode(ids) == want
        out_ids = []
        for t in reply[:n]:
            out_ids.append(t)
            if stop_fn is not None and stop_fn(out_ids):
                return out_ids, "stop"
        return out_ids, "length"
    monkeypatch.setattr(serve, "sample", fake_sample)
    st, out = srv.handle_request("POST", "/v1/chat/completions", json.dumps(dict(body, max_tokens=40)).encode())
    assert out["choices"][0]["message"]["content"] == "Hello!" and out["choices"][0]["finish_reason"] == "stop"
    assert out["usage"]["completion_tokens"] == len(tok.encode("Hello!<|im_end|>"))
    # invalid: no messages, unknown role, unknown template
    for bad in ({"messages": []}, {"messages": [{"role": "robot", "content": "x"}]},
                {"messages": [{"role": "user", "content": "x"}], "template": "alpaca"}):
        assert srv.handle_request("POST", "/v1/chat/completions", json.dumps(bad).encode())[0] == 400
    # without a tokenizer chat is refused
    srv2 = serve.CompletionServer(str(tmp_path / "model.safetensors"), "cpu", max_tokens_cap=8)
    assert srv2.handle_request("POST", "/v1/chat/completions", json.dumps(body).encode())[0] == 400
