"""Model architecture descriptions and the presets served by this runtime.

The reference runtime learns geometry from ``config.json`` / ONNX
``past_key_values.*`` shapes (crates/kapsl-llm/src/engine.rs:1823-1994); here
the same fields are read from HF ``config.json`` or GGUF metadata
(:mod:`kapsl_sdk_b200.loaders`) into :class:`ModelConfig`.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import asdict, dataclass, field
from typing import Optional


# HF model_type -> the runtime's layer family (Mistral and Phi-3 are Llama-shaped
# decoders; Phi-3's fused projections are split by the checkpoint loader)
HF_MODEL_TYPES = {"llama": "llama", "mistral": "llama", "phi3": "llama", "qwen2": "qwen2", "mixtral": "mixtral",
                  "qwen3": "qwen3", "gemma": "gemma", "gemma2": "gemma2"}


@dataclass
class ModelConfig:
    name: str = "custom"
    arch: str = "llama"  # llama | qwen2 | qwen3 | mixtral | gemma | gemma2
    vocab_size: int = 32000
    hidden_size: int = 4096
    intermediate_size: int = 11008
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: int = 32
    head_dim: int = 128
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5
    qkv_bias: bool = False
    tie_embeddings: bool = False
    max_position: int = 32768
    num_experts: int = 0
    experts_per_token: int = 0
    weight_format: str = "bf16"  # bf16 | q4_k (GGUF k-quant linear layers, dequantized in the GEMM)
    rope_scaling: Optional[dict] = None  # HF rope_scaling (linear | llama3 | yarn) or GGUF frequency factors
    qk_norm: bool = False  # per-head RMSNorm of q and k before RoPE (Qwen3); CPU backend only
    # Gemma-family options (CPU backend only)
    act: str = "silu"              # gated-MLP activation: silu | gelu_tanh
    embed_scale: float = 1.0       # token embeddings multiplied by this (Gemma: sqrt(hidden))
    attn_scale: Optional[float] = None  # attention logit scale (default 1/sqrt(head_dim))
    attn_softcap: float = 0.0      # logits -> cap * tanh(logits / cap) when > 0
    final_softcap: float = 0.0
    sliding_window: int = 0        # local attention window of the sliding layers
    sliding_pattern: int = 0       # layer i is sliding iff i % pattern != pattern - 1 (0: none)
    layer_types: Optional[list] = None  # explicit "sliding_attention" / "full_attention" per layer

    def layer_window(self, i: int) -> int:
        """Key window of layer ``i`` (0: full causal attention)."""
        if not self.sliding_window:
            return 0
        if self.layer_types:
            return self.sliding_window if self.layer_types[i] == "sliding_attention" else 0
        if self.sliding_pattern and i % self.sliding_pattern != self.sliding_pattern - 1:
            return self.sliding_window
        return 0

    @property
    def cpu_only(self) -> bool:
        """Features the GPU kernels do not implement."""
        return (self.qk_norm or self.act != "silu" or self.embed_scale != 1.0 or self.attn_scale is not None or
                self.attn_softcap > 0 or self.final_softcap > 0 or self.sliding_pattern > 0 or
                bool(self.layer_types))
    bos_token_id: Optional[int] = 1
    eos_token_id: Optional[int] = 2
    extra: dict = field(default_factory=dict)

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        """Bytes of K+V for one token over all layers (reference: L*H_kv*D*2*2, engine.rs:2144)."""
        return self.num_layers * self.num_kv_heads * self.head_dim * 2 * dtype_bytes

    def num_params(self) -> int:
        d, f, L = self.hidden_size, self.intermediate_size, self.num_layers
        attn = d * (self.q_size + 2 * self.kv_size) + self.q_size * d
        mlp = 3 * d * f * (self.num_experts if self.is_moe else 1) + (d * self.num_experts if self.is_moe else 0)
        emb = self.vocab_size * d * (1 if self.tie_embeddings else 2)
        return L * (attn + mlp + 2 * d) + emb + d

    def active_params(self) -> int:
        """Parameters touched per token (MoE: only the routed experts)."""
        if not self.is_moe:
            return self.num_params()
        d, f, L = self.hidden_size, self.intermediate_size, self.num_layers
        attn = d * (self.q_size + 2 * self.kv_size) + self.q_size * d
        mlp = 3 * d * f * self.experts_per_token + d * self.num_experts
        emb = self.vocab_size * d * (1 if self.tie_embeddings else 2)
        return L * (attn + mlp + 2 * d) + emb + d

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_hf_config(cls, path_or_dict) -> "ModelConfig":
        """Build from a HuggingFace ``config.json`` (path or dict)."""
        if isinstance(path_or_dict, (str, os.PathLike)):
            with open(path_or_dict) as f:
                c = json.load(f)
        else:
            c = dict(path_or_dict)
        mt = c.get("model_type", "llama")
        rp = c.get("rope_parameters")  # transformers >= 5 keeps rope_theta and the scaling here
        if isinstance(rp, dict) and "rope_theta" in rp:
            c.setdefault("rope_theta", rp["rope_theta"])
            if rp.get("rope_type", "default") != "default" and not c.get("rope_scaling"):
                c["rope_scaling"] = {k: v for k, v in rp.items() if k != "rope_theta"}
        if mt not in HF_MODEL_TYPES:
            raise ValueError(f"model_type {mt!r} is not supported (supported: {', '.join(sorted(HF_MODEL_TYPES))})")
        arch = HF_MODEL_TYPES[mt]
        if float(c.get("partial_rotary_factor", 1.0)) != 1.0:
            raise ValueError("partial rotary embeddings are not supported")
        heads = c.get("num_attention_heads", 32)
        hidden = c.get("hidden_size", 4096)
        max_pos = int(c.get("max_position_embeddings", 32768))
        window = c.get("sliding_window") if c.get("use_sliding_window", True) else None
        gemma = {}
        if mt in ("gemma", "gemma2"):
            act = c.get("hidden_activation") or c.get("hidden_act") or "gelu_pytorch_tanh"
            if act not in ("gelu_pytorch_tanh", "gelu"):
                raise ValueError(f"Gemma activation {act!r} is not supported")
            gemma = dict(act="gelu_tanh", embed_scale=math.sqrt(hidden))
            if mt == "gemma2":
                gemma.update(attn_softcap=float(c.get("attn_logit_softcapping") or 0.0),
                             final_softcap=float(c.get("final_logit_softcapping") or 0.0),
                             attn_scale=float(c.get("query_pre_attn_scalar", c.get("head_dim", 256))) ** -0.5,
                             sliding_window=int(window or 0), sliding_pattern=2 if window else 0,
                             layer_types=list(c["layer_types"]) if c.get("layer_types") else None)
            window = None  # handled per layer
        if window and int(window) < max_pos:
            # sliding-window attention equals full attention up to the window: serve that far exactly
            max_pos = int(window)
        eos = c.get("eos_token_id")
        if isinstance(eos, list):
            eos = eos[0] if eos else None
        return cls(
            name=c.get("_name_or_path", mt),
            arch=arch,
            vocab_size=c.get("vocab_size", 32000),
            hidden_size=hidden,
            intermediate_size=c.get("intermediate_size", 4 * hidden),
            num_layers=c.get("num_hidden_layers", 32),
            num_heads=heads,
            num_kv_heads=c.get("num_key_value_heads", heads),
            head_dim=c.get("head_dim", hidden // heads),
            rope_theta=float(c.get("rope_theta", 10000.0)),
            rms_eps=float(c.get("rms_norm_eps", 1e-5)),
            qkv_bias=bool(c.get("attention_bias", arch == "qwen2")),
            tie_embeddings=bool(c.get("tie_word_embeddings", mt in ("gemma", "gemma2"))),
            max_position=max_pos,
            num_experts=int(c.get("num_local_experts", 0)),
            experts_per_token=int(c.get("num_experts_per_tok", 0)),
            bos_token_id=c.get("bos_token_id"),
            eos_token_id=eos,
            rope_scaling=_rope_scaling(c),
            qk_norm=mt == "qwen3",
            **gemma,
        )


def _rope_scaling(c: dict) -> Optional[dict]:
    """HF ``rope_scaling`` (older configs name the kind ``type``), with the
    original context length defaulted from the config; the check happens here
    so an unsupported kind fails at load time."""
    rs = c.get("rope_scaling")
    if not rs:
        return None
    rs = dict(rs)
    kind = rs.get("rope_type", rs.get("type", "default"))
    rs["rope_type"] = kind
    if kind == "default":
        return None
    if kind in ("yarn", "llama3"):
        rs.setdefault("original_max_position_embeddings", c.get("original_max_position_embeddings",
                                                                c.get("max_position_embeddings", 4096)))
    from ..ops.reference import rope_inv_freq

    rope_inv_freq(c.get("head_dim", c.get("hidden_size", 4096) // c.get("num_attention_heads", 32)),
                  float(c.get("rope_theta", 10000.0)), rs)
    return rs


def tiny_llama() -> ModelConfig:
    """4 layers, d 512, 8/8 heads of 64, FFN 1408, vocab 32000 (CPU GGUF workload)."""
    return ModelConfig(name="tiny-llama", arch="llama", vocab_size=32000, hidden_size=512, intermediate_size=1408,
                       num_layers=4, num_heads=8, num_kv_heads=8, head_dim=64, rope_theta=10000.0, rms_eps=1e-5,
                       max_position=4096)


def tiny_qwen2() -> ModelConfig:
    """2 layers, d 512, 8q/2kv heads of 128, FFN 1024, vocab 4096, QKV bias: the smallest
    Qwen2-style decoder the GPU kernels take (head dim 128), for smoke runs and tests."""
    return ModelConfig(name="tiny-qwen2", arch="qwen2", vocab_size=4096, hidden_size=512, intermediate_size=1024,
                       num_layers=2, num_heads=8, num_kv_heads=2, head_dim=128, rope_theta=1e6, rms_eps=1e-6,
                       qkv_bias=True, max_position=4096)


def qwen2_5_7b() -> ModelConfig:
    """Qwen2.5-7B: 28 layers, d 3584, 28q/4kv heads of 128, FFN 18944, vocab 152064, theta 1e6, QKV bias."""
    return ModelConfig(name="qwen2.5-7b", arch="qwen2", vocab_size=152064, hidden_size=3584, intermediate_size=18944,
                       num_layers=28, num_heads=28, num_kv_heads=4, head_dim=128, rope_theta=1e6, rms_eps=1e-6,
                       qkv_bias=True, max_position=32768, bos_token_id=151643, eos_token_id=151645)


def llama3_70b() -> ModelConfig:
    """Llama-3-70B: 80 layers, d 8192, 64q/8kv heads of 128, FFN 28672, vocab 128256, theta 5e5."""
    return ModelConfig(name="llama-3-70b", arch="llama", vocab_size=128256, hidden_size=8192, intermediate_size=28672,
                       num_layers=80, num_heads=64, num_kv_heads=8, head_dim=128, rope_theta=5e5, rms_eps=1e-5,
                       max_position=8192, bos_token_id=128000, eos_token_id=128001)


def llama3_8b() -> ModelConfig:
    """Llama-3-8B: 32 layers, d 4096, 32q/8kv heads of 128, FFN 14336, vocab 128256, theta 5e5."""
    return ModelConfig(name="llama-3-8b", arch="llama", vocab_size=128256, hidden_size=4096, intermediate_size=14336,
                       num_layers=32, num_heads=32, num_kv_heads=8, head_dim=128, rope_theta=5e5, rms_eps=1e-5,
                       max_position=16384, bos_token_id=128000, eos_token_id=128001)


def mixtral_8x7b() -> ModelConfig:
    """Mixtral-8x7B: 32 layers, d 4096, 32q/8kv heads, 8 experts top-2, expert FFN 14336, vocab 32000."""
    return ModelConfig(name="mixtral-8x7b", arch="mixtral", vocab_size=32000, hidden_size=4096,
                       intermediate_size=14336, num_layers=32, num_heads=32, num_kv_heads=8, head_dim=128,
                       rope_theta=1e6, rms_eps=1e-5, max_position=32768, num_experts=8, experts_per_token=2)


def llama3_70b_q4k() -> ModelConfig:
    """Llama-3-70B with GGUF Q4_K linear layers (embedding / lm_head kept bf16)."""
    cfg = llama3_70b()
    cfg.name = "llama-3-70b-q4k"
    cfg.weight_format = "q4_k"
    return cfg


PRESETS = {
    "tiny-llama": tiny_llama,
    "tiny-qwen2": tiny_qwen2,
    "qwen2.5-7b": qwen2_5_7b,
    "llama-3-70b": llama3_70b,
    "llama-3-70b-q4k": llama3_70b_q4k,
    "llama-3-8b": llama3_8b,
    "mixtral-8x7b": mixtral_8x7b,
}


def get_preset(name: str, **overrides) -> ModelConfig:
    cfg = PRESETS[name]()
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg
