"""RoPE scaling: the rotary tables for linear, Llama-3 and YaRN scaling match
transformers' RoPE initialisers; configs carry the scaling from HF
config.json and GGUF metadata; an engine on a scaled model matches the dense
fp32 oracle built from the same table."""
import math
import os
import tempfile

import pytest
import torch

from kapsl_sdk_b200.models.config import ModelConfig
from kapsl_sdk_b200.ops import reference as ref


def _hf(kind_cfg: dict, head_dim=64, theta=500000.0, max_pos=131072):
    from transformers import LlamaConfig
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    c = LlamaConfig(hidden_size=head_dim * 4, num_attention_heads=4, num_key_value_heads=2, head_dim=head_dim,
                    rope_theta=theta, max_position_embeddings=max_pos, rope_scaling=dict(kind_cfg))
    kind = kind_cfg["rope_type"]
    inv, attn = ROPE_INIT_FUNCTIONS[kind](c, torch.device("cpu"))
    return inv.double(), float(attn)


@pytest.mark.parametrize("rs", [
    {"rope_type": "linear", "factor": 4.0},
    {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
     "original_max_position_embeddings": 8192},
    {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 32768},
    {"rope_type": "yarn", "factor": 16.0, "original_max_position_embeddings": 4096, "beta_fast": 16.0,
     "beta_slow": 2.0},
])
def test_inverse_frequencies_match_transformers(rs):
    try:
        want_inv, want_attn = _hf(rs)
    except Exception as e:  # pragma: no cover - transformers API drift
        pytest.skip(f"transformers RoPE initialiser unavailable: {e}")
    inv, attn = ref.rope_inv_freq(64, 500000.0, rs)
    assert torch.allclose(inv, want_inv, rtol=1e-6, atol=0)
    assert math.isclose(attn, want_attn, rel_tol=1e-9)


def test_table_and_refusals():
    base = ref.rope_cos_sin(16, 8, 10000.0)
    lin = ref.rope_cos_sin(16, 8, 10000.0, scaling={"rope_type": "linear", "factor": 2.0})
    assert torch.allclose(lin[2], base[1])  # position 2 at half speed == position 1
    y = ref.rope_cos_sin(4, 8, 10000.0, scaling={"rope_type": "yarn", "factor": 4.0,
                                                  "original_max_position_embeddings": 64})
    assert math.isclose(y[0, 0].item(), 0.1 * math.log(4.0) + 1.0, rel_tol=1e-6)  # cos(0) * attention factor
    ff = ref.rope_cos_sin(16, 8, 10000.0, scaling={"rope_type": "freq_factors", "factors": [1.0, 1.0, 2.0, 4.0]})
    inv, _ = ref.rope_inv_freq(8, 10000.0)
    assert torch.allclose(ff[5, 3], torch.tensor(math.cos(5 * inv[3].item() / 4.0), dtype=torch.float32))
    for kind in ("dynamic", "longrope"):
        with pytest.raises(ValueError, match="live sequence length"):
            ref.rope_inv_freq(8, 10000.0, {"rope_type": kind, "factor": 2.0})
    with pytest.raises(ValueError, match="live sequence length"):
        ModelConfig.from_hf_config({"rope_scaling": {"type": "dynamic", "factor": 2.0}})


def test_configs_carry_scaling_through_hf_and_gguf():
    from kapsl_sdk_b200.loaders.gguf import gguf_config, write_gguf_model
    from kapsl_sdk_b200.models.llama import random_full_weights

    c = ModelConfig.from_hf_config({"model_type": "llama", "hidden_size": 256, "num_attention_heads": 4,
                                    "max_position_embeddings": 2048,
                                    "rope_scaling": {"type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                                     "high_freq_factor": 4.0}})
    assert c.rope_scaling["rope_type"] == "llama3"
    assert c.rope_scaling["original_max_position_embeddings"] == 2048
    from gguf import GGUFReader

    cfg = ModelConfig(name="g", vocab_size=300, hidden_size=64, intermediate_size=128, num_layers=1, num_heads=4,
                      num_kv_heads=2, head_dim=16, max_position=256,
                      rope_scaling={"rope_type": "freq_factors", "factors": [1.0] * 4 + [3.0] * 4})
    d = tempfile.mkdtemp()
    for rs in (cfg.rope_scaling, {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 64}):
        cfg.rope_scaling = rs
        p = os.path.join(d, "m.gguf")
        write_gguf_model(p, cfg, random_full_weights(cfg, torch.device("cpu"), seed=0), quant="f32")
        got = gguf_config(GGUFReader(p)).rope_scaling
        assert got["rope_type"] == rs["rope_type"]
        if rs["rope_type"] == "freq_factors":
            assert got["factors"] == rs["factors"]
        else:
            assert got["factor"] == 4.0 and got["original_max_position_embeddings"] == 64


def test_scaled_model_engine_matches_dense_oracle():
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.llama import reference_forward

    cfg = ModelConfig(name="t", vocab_size=300, hidden_size=64, intermediate_size=128, num_layers=2, num_heads=4,
                      num_kv_heads=2, head_dim=16, max_position=512, bos_token_id=None, eos_token_id=None,
                      rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                    "high_freq_factor": 4.0, "original_max_position_embeddings": 64})
    eng = LLMEngine(cfg, device="cpu", engine_cfg=EngineConfig(max_num_seqs=2, max_num_batched_tokens=32,
                                                                max_model_len=256, num_blocks=64), seed=0)
    prompt = list(range(5, 105))
    out = eng.generate([prompt], SamplingParams.greedy(5, ignore_eos=True))[0]
    m = eng.model
    toks = list(prompt)
    for _ in range(5):
        toks.append(int(reference_forward(cfg, m.layers, m.embed, m.lm_head, m.final_norm, toks)[-1].argmax()))
    assert out == toks[len(prompt):]
    assert not torch.allclose(m.cos_sin, ref.rope_cos_sin(cfg.max_position, 16, cfg.rope_theta))
