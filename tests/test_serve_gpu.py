"""Generation on the CUDA engine: next-token logits against the fp32 oracle, and the completion server
answering on a GPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model(tmp_path):
    from distrain_b200.config import ModelConfig
    from distrain_b200.models.params import ParamLayout, init_flat
    from distrain_b200.utils.checkpoint import save_safetensors
    cfg = ModelConfig(hidden_dim=128, num_layers=2, num_heads=4, num_kv_heads=2, ffn_hidden_dim=256, vocab_size=512,
                      max_seq_len=256, rope_theta=10000.0)
    L = ParamLayout(cfg)
    sd = L.to_state_dict(init_flat(L, 0.08, 5))
    path = str(tmp_path / "m.safetensors")
    save_safetensors(sd, path)
    return cfg, sd, path


def test_engine_logits_match_oracle(tmp_path):
    from distrain_b200.models import oracle
    from distrain_b200.serve import EngineLM
    cfg, sd, _ = _model(tmp_path)
    W = 300  # windows 128, 256 and 300
    lm = EngineLM(sd, cfg, "cuda:0", window=W)
    g = torch.Generator().manual_seed(0)
    for n in (1, 7, 128, 130, 256, 300, 400):  # 400 > window: the last 300 tokens are the context
        seq = torch.randint(0, 512, (n,), generator=g).tolist()
        z = lm.next_logits(seq)
        ctx = torch.tensor([seq[-W:]])
        ref = oracle.logits_fn({k: v.float() for k, v in sd.items()}, cfg, ctx, mask_value=None)[0, -1]
        rel = ((z - ref).norm() / ref.norm()).item()
        assert rel < 3e-2, (n, rel)
    # one engine per window, all on the same weights
    assert sorted(lm.engines) == [128, 256, 300]
    assert all(e.master.data_ptr() == lm.eng.master.data_ptr() and e.p16.data_ptr() == lm.eng.p16.data_ptr()
               for e in lm.engines.values())


def test_completion_server_on_gpu(tmp_path):
    from distrain_b200.serve import CompletionServer
    _, _, path = _model(tmp_path)
    srv = CompletionServer(path, device="cuda:0", max_tokens_cap=32)
    assert srv.lm is not None
    code, body = srv.complete({"prompt": [1, 2, 3, 4], "max_tokens": 8})
    assert code == 200
    assert len(body["choices"][0]["token_ids"]) == 8 and body["usage"]["total_tokens"] == 12
    code2, body2 = srv.complete({"prompt": [1, 2, 3, 4], "max_tokens": 8})
    assert body2["choices"][0]["token_ids"] == body["choices"][0]["token_ids"]  # greedy is deterministic
