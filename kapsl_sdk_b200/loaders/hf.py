"""HuggingFace checkpoints (``config.json`` + ``*.safetensors``) for the
Llama / Mistral / Qwen2 / Mixtral / Phi-3 families.

Tensor names ``model.embed_tokens.weight``, ``lm_head.weight``, ``model.norm.weight``,
``model.layers.{i}.{input_layernorm, post_attention_layernorm}.weight``,
``self_attn.{q,k,v,o}_proj.{weight,bias}``, ``mlp.{gate,up,down}_proj.weight`` and,
for Mixtral, ``block_sparse_moe.gate.weight`` / ``experts.{e}.w{1,3,2}.weight``
are mapped to this runtime's full-tensor stream, then sharded per rank.  Phi-3's
fused ``self_attn.qkv_proj`` and ``mlp.gate_up_proj`` are split into the same
tensors.
"""
from __future__ import annotations

import glob
import json
import os

import torch

from ..models.config import ModelConfig


class _SafeTensors:
    def __init__(self, root: str):
        from safetensors import safe_open

        self.files = sorted(glob.glob(os.path.join(root, "*.safetensors")))
        if not self.files:
            raise FileNotFoundError(f"no .safetensors files in {root}")
        self.where = {}
        self.handles = [safe_open(f, framework="pt") for f in self.files]
        for h in self.handles:
            for k in h.keys():
                self.where[k] = h

    def get(self, name: str) -> torch.Tensor:
        return self.where[name].get_tensor(name)

    def has(self, name: str) -> bool:
        return name in self.where


def iter_hf_full(root: str, cfg: ModelConfig):
    st = _SafeTensors(root)
    gemma = cfg.arch in ("gemma", "gemma2")

    def norm(name):  # Gemma stores w for a (1 + w) RMSNorm scale
        w = st.get(name)
        return w.float() + 1.0 if gemma else w

    emb = st.get("model.embed_tokens.weight")
    yield "embed", emb
    yield "lm_head", st.get("lm_head.weight") if st.has("lm_head.weight") else emb
    yield "final_norm", norm("model.norm.weight")
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        a = p + "self_attn."
        full = {"o": st.get(a + "o_proj.weight"), "in_norm": norm(p + "input_layernorm.weight")}
        if cfg.arch == "gemma2":  # sandwich norms around attention and MLP
            full["attn_out_norm"] = norm(p + "post_attention_layernorm.weight")
            full["post_norm"] = norm(p + "pre_feedforward_layernorm.weight")
            full["mlp_out_norm"] = norm(p + "post_feedforward_layernorm.weight")
        else:
            full["post_norm"] = norm(p + "post_attention_layernorm.weight")
        if st.has(a + "qkv_proj.weight"):  # Phi-3: fused [q; k; v]
            full["q"], full["k"], full["v"] = torch.split(st.get(a + "qkv_proj.weight"),
                                                          [cfg.q_size, cfg.kv_size, cfg.kv_size], 0)
        else:
            full["q"], full["k"], full["v"] = (st.get(a + "q_proj.weight"), st.get(a + "k_proj.weight"),
                                               st.get(a + "v_proj.weight"))
        if st.has(a + "q_norm.weight"):  # Qwen3
            full["q_norm"], full["k_norm"] = st.get(a + "q_norm.weight"), st.get(a + "k_norm.weight")
        if st.has(a + "q_proj.bias"):
            full["q_b"], full["k_b"], full["v_b"] = (st.get(a + "q_proj.bias"), st.get(a + "k_proj.bias"),
                                                   st.get(a + "v_proj.bias"))
        if cfg.is_moe:
            m = p + "block_sparse_moe."
            full["router"] = st.get(m + "gate.weight")
            full["experts_gate"] = torch.stack([st.get(f"{m}experts.{e}.w1.weight") for e in range(cfg.num_experts)])
            full["experts_up"] = torch.stack([st.get(f"{m}experts.{e}.w3.weight") for e in range(cfg.num_experts)])
            full["experts_down"] = torch.stack([st.get(f"{m}experts.{e}.w2.weight") for e in range(cfg.num_experts)])
        elif st.has(p + "mlp.gate_up_proj.weight"):  # Phi-3: fused [gate; up]
            full["gate"], full["up"] = torch.chunk(st.get(p + "mlp.gate_up_proj.weight"), 2, 0)
            full["down"] = st.get(p + "mlp.down_proj.weight")
        else:
            full["gate"] = st.get(p + "mlp.gate_proj.weight")
            full["up"] = st.get(p + "mlp.up_proj.weight")
            full["down"] = st.get(p + "mlp.down_proj.weight")
        yield "layer", full


def load_hf_model(root: str, device, tp: int = 1, rank: int = 0):
    from ..models.cpu_model import CPUCausalLM
    from ..models.llama import weights_from_full

    cfg = ModelConfig.from_hf_config(os.path.join(root, "config.json"))
    dev = torch.device(device)
    stream = iter_hf_full(root, cfg)
    if dev.type == "cpu":
        items = list(stream)
        d = dict((k, v) for k, v in items if k != "layer")
        return cfg, CPUCausalLM(cfg, d["embed"], d["lm_head"], d["final_norm"],
                                [v for k, v in items if k == "layer"]), None
    conv = ((k, v.to(dev, torch.bfloat16) if isinstance(v, torch.Tensor)
             else {kk: vv.to(dev, torch.bfloat16) for kk, vv in v.items()}) for k, v in stream)
    return cfg, weights_from_full(cfg, conv, dev, tp, rank), None


def save_hf_model(root: str, cfg: ModelConfig, full_stream) -> None:
    """Write a full-tensor stream as a HF-style checkpoint (one safetensors file)."""
    from safetensors.torch import save_file

    os.makedirs(root, exist_ok=True)
    t = {}
    li = 0
    for kind, v in full_stream:
        if kind == "embed":
            t["model.embed_tokens.weight"] = v
        elif kind == "lm_head":
            t["lm_head.weight"] = v
        elif kind == "final_norm":
            t["model.norm.weight"] = v
        else:
            p = f"model.layers.{li}."
            a = p + "self_attn."
            t[a + "q_proj.weight"], t[a + "k_proj.weight"], t[a + "v_proj.weight"] = v["q"], v["k"], v["v"]
            t[a + "o_proj.weight"] = v["o"]
            t[p + "input_layernorm.weight"] = v["in_norm"]
            t[p + "post_attention_layernorm.weight"] = v["post_norm"]
            if v.get("q_b") is not None:
                t[a + "q_proj.bias"], t[a + "k_proj.bias"], t[a + "v_proj.bias"] = v["q_b"], v["k_b"], v["v_b"]
            if v.get("q_norm") is not None:
                t[a + "q_norm.weight"], t[a + "k_norm.weight"] = v["q_norm"], v["k_norm"]
            if "gate" in v:
                t[p + "mlp.gate_proj.weight"], t[p + "mlp.up_proj.weight"] = v["gate"], v["up"]
                t[p + "mlp.down_proj.weight"] = v["down"]
            li += 1
    t.setdefault("model.norm.weight", torch.ones(cfg.hidden_size))
    save_file({k: x.detach().contiguous().cpu() for k, x in t.items()}, os.path.join(root, "model.safetensors"))
    hf = {"model_type": "qwen3" if cfg.qk_norm else ("qwen2" if cfg.arch == "qwen2" else "llama"),
          "vocab_size": cfg.vocab_size,
          "hidden_size": cfg.hidden_size, "intermediate_size": cfg.intermediate_size,
          "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.num_heads,
          "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim, "rope_theta": cfg.rope_theta,
          "rms_norm_eps": cfg.rms_eps, "attention_bias": cfg.qkv_bias, "tie_word_embeddings": cfg.tie_embeddings,
          "max_position_embeddings": cfg.max_position, "bos_token_id": cfg.bos_token_id,
          "eos_token_id": cfg.eos_token_id}
    if cfg.rope_scaling:
        hf["rope_scaling"] = dict(cfg.rope_scaling)
    with open(os.path.join(root, "config.json"), "w") as f:
        json.dump(hf, f)
