"""Export a checkpoint to the Hugging Face ``Qwen2ForCausalLM`` layout, for evaluation and serving tools
of that ecosystem.

The architecture maps one to one: pre-norm GQA decoder, bias on the q/k/v projections only, rotate-half
RoPE, RMSNorm, SwiGLU, tied input/output embedding. The one extra is the learned scalar
``embedding.output_scale`` that multiplies the final hidden state before the tied head
(logits = (norm(h) * s) E^T); it is folded into the final norm's weight. A checkpoint without q/k/v bias
gets zero biases. The reference's export script (scripts/export_hf.py) depends on a package that is not
in its repository; this is a working counterpart with a logit-level check against the fp32 oracle
(tests/test_hf_export_cpu.py)."""
from __future__ import annotations

import json
import os
from typing import Dict

import torch

from ..config import ModelConfig


def hf_config(cfg: ModelConfig) -> dict:
    return {
        "architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2",
        "vocab_size": cfg.vocab_size, "hidden_size": cfg.hidden_dim, "intermediate_size": cfg.ffn_hidden_dim,
        "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.num_heads,
        "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.hidden_dim // cfg.num_heads,
        "max_position_embeddings": cfg.max_seq_len, "rms_norm_eps": cfg.norm_eps, "rope_theta": cfg.rope_theta,
        "rope_parameters": {"rope_type": "default", "rope_theta": cfg.rope_theta},
        "hidden_act": "silu", "tie_word_embeddings": True, "attention_dropout": 0.0, "use_sliding_window": False,
        "torch_dtype": "float32",
    }


def to_hf_state_dict(sd: Dict[str, torch.Tensor], cfg: ModelConfig) -> Dict[str, torch.Tensor]:
    out = {"model.embed_tokens.weight": sd["embedding.embedding.weight"].float()}
    d = cfg.hidden_dim // cfg.num_heads
    sizes = {"q_proj": cfg.num_heads * d, "k_proj": cfg.num_kv_heads * d, "v_proj": cfg.num_kv_heads * d}
    for i in range(cfg.num_layers):
        src, dst = f"layers.{i}", f"model.layers.{i}"
        out[f"{dst}.input_layernorm.weight"] = sd[f"{src}.attn_norm.weight"].float()
        out[f"{dst}.post_attention_layernorm.weight"] = sd[f"{src}.ffn_norm.weight"].float()
        for proj, n in sizes.items():
            out[f"{dst}.self_attn.{proj}.weight"] = sd[f"{src}.attention.{proj}.weight"].float()
            b = sd.get(f"{src}.attention.{proj}.bias")
            out[f"{dst}.self_attn.{proj}.bias"] = b.float() if b is not None else torch.zeros(n)
        out[f"{dst}.self_attn.o_proj.weight"] = sd[f"{src}.attention.o_proj.weight"].float()
        for proj in ("gate_proj", "up_proj", "down_proj"):
            out[f"{dst}.mlp.{proj}.weight"] = sd[f"{src}.ffn.{proj}.weight"].float()
    scale = sd["embedding.output_scale"].float().reshape(-1)[0]
    out["model.norm.weight"] = sd["final_norm.weight"].float() * scale
    return {k: v.contiguous() for k, v in out.items()}


def export_hf(sd: Dict[str, torch.Tensor], cfg: ModelConfig, out_dir: str) -> str:
    """Write ``config.json`` and ``model.safetensors`` (fp32) into ``out_dir``."""
    from .checkpoint import save_safetensors
    os.makedirs(out_dir, exist_ok=True)
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(hf_config(cfg), f, indent=2)
    with open(os.path.join(out_dir, "model.safetensors"), "wb") as f:
        f.write(save_safetensors(to_hf_state_dict(sd, cfg)))
    return out_dir


def from_hf(hf_dir: str):
    """A Hugging Face ``Qwen2ForCausalLM``-layout directory (config.json + safetensors) -> (state dict in
    this framework's layout, ModelConfig), e.g. to start training from a pretrained model. Requires tied
    embeddings and head_dim = hidden / heads; the output scale is 1 (the final norm keeps the weight)."""
    import glob
    from .checkpoint import load_safetensors
    with open(os.path.join(hf_dir, "config.json")) as f:
        c = json.load(f)
    if c.get("model_type") not in ("qwen2", None) and "Qwen2ForCausalLM" not in c.get("architectures", []):
        raise ValueError(f"not a Qwen2-layout model: {c.get('model_type')}")
    H, nh = int(c["hidden_size"]), int(c["num_attention_heads"])
    if int(c.get("head_dim") or H // nh) * nh != H:
        raise ValueError("head_dim * heads must equal the hidden size")
    rope = c.get("rope_parameters") or {}
    cfg = ModelConfig(hidden_dim=H, num_layers=int(c["num_hidden_layers"]), num_heads=nh,
                      num_kv_heads=int(c.get("num_key_value_heads", nh)), ffn_hidden_dim=int(c["intermediate_size"]),
                      vocab_size=int(c["vocab_size"]), max_seq_len=int(c.get("max_position_embeddings", 4096)),
                      rope_theta=float(rope.get("rope_theta", c.get("rope_theta", 10000.0))),
                      norm_eps=float(c.get("rms_norm_eps", 1e-6)), qkv_bias=True)
    hf = {}
    for f in sorted(glob.glob(os.path.join(hf_dir, "*.safetensors"))):
        hf.update(load_safetensors(f))
    if "lm_head.weight" in hf and not torch.equal(hf["lm_head.weight"], hf["model.embed_tokens.weight"]):
        raise ValueError("untied output head: this architecture ties the head to the embedding")
    if not c.get("tie_word_embeddings", True):
        raise ValueError("tie_word_embeddings is false: this architecture ties the head to the embedding")
    sd = {"embedding.embedding.weight": hf["model.embed_tokens.weight"].float(),
          "embedding.output_scale": torch.ones(1), "final_norm.weight": hf["model.norm.weight"].float()}
    for i in range(cfg.num_layers):
        src, dst = f"model.layers.{i}", f"layers.{i}"
        sd[f"{dst}.attn_norm.weight"] = hf[f"{src}.input_layernorm.weight"].float()
        sd[f"{dst}.ffn_norm.weight"] = hf[f"{src}.post_attention_layernorm.weight"].float()
        for proj in ("q_proj", "k_proj", "v_proj"):
            sd[f"{dst}.attention.{proj}.weight"] = hf[f"{src}.self_attn.{proj}.weight"].float()
            sd[f"{dst}.attention.{proj}.bias"] = hf[f"{src}.self_attn.{proj}.bias"].float()
        sd[f"{dst}.attention.o_proj.weight"] = hf[f"{src}.self_attn.o_proj.weight"].float()
        for proj in ("gate_proj", "up_proj", "down_proj"):
            sd[f"{dst}.ffn.{proj}.weight"] = hf[f"{src}.mlp.{proj}.weight"].float()
    return sd, cfg
