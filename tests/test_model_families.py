"""Model families served through the Llama-shaped decoder: Mistral (sliding
window capped to the window), Phi-3 (fused qkv / gate_up projections, in HF
and GGUF checkpoints); unsupported families are refused at load time."""
import json
import os
import tempfile

import pytest
import torch

from kapsl_sdk_b200.models.config import ModelConfig


def tiny():
    return ModelConfig(name="t", arch="llama", vocab_size=300, hidden_size=64, intermediate_size=128, num_layers=2,
                       num_heads=4, num_kv_heads=2, head_dim=16, max_position=256, bos_token_id=None,
                       eos_token_id=None)


def _greedy(model_cfg, model, prompt):
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams

    eng = LLMEngine(model_cfg, weights=model, device="cpu", engine_cfg=EngineConfig(
        max_num_seqs=2, max_num_batched_tokens=64, max_model_len=200, num_blocks=32), seed=0)
    return eng.generate([prompt], SamplingParams.greedy(6, ignore_eos=True))[0]


def test_phi3_hf_checkpoint_matches_unfused_llama():
    from safetensors.torch import load_file, save_file

    from kapsl_sdk_b200.loaders.hf import load_hf_model, save_hf_model
    from kapsl_sdk_b200.models.llama import random_full_weights

    cfg = tiny()
    d = tempfile.mkdtemp()
    llama, phi = os.path.join(d, "llama"), os.path.join(d, "phi3")
    save_hf_model(llama, cfg, random_full_weights(cfg, torch.device("cpu"), seed=3, std=0.1))
    t = load_file(os.path.join(llama, "model.safetensors"))
    for i in range(cfg.num_layers):
        a, m = f"model.layers.{i}.self_attn.", f"model.layers.{i}.mlp."
        t[a + "qkv_proj.weight"] = torch.cat([t.pop(a + "q_proj.weight"), t.pop(a + "k_proj.weight"),
                                              t.pop(a + "v_proj.weight")], 0)
        t[m + "gate_up_proj.weight"] = torch.cat([t.pop(m + "gate_proj.weight"), t.pop(m + "up_proj.weight")], 0)
    os.makedirs(phi)
    save_file(t, os.path.join(phi, "model.safetensors"))
    c = json.load(open(os.path.join(llama, "config.json")))
    c["model_type"] = "phi3"
    json.dump(c, open(os.path.join(phi, "config.json"), "w"))
    cfg_l, m_l, _ = load_hf_model(llama, "cpu")
    cfg_p, m_p, _ = load_hf_model(phi, "cpu")
    prompt = list(range(7, 60))
    assert _greedy(cfg_p, m_p, prompt) == _greedy(cfg_l, m_l, prompt)


def test_phi3_gguf_matches_llama_gguf():
    from kapsl_sdk_b200.loaders.gguf import load_gguf_model, write_gguf_model
    from kapsl_sdk_b200.models.llama import random_full_weights

    cfg = tiny()
    d = tempfile.mkdtemp()
    outs = []
    for arch in ("llama", "phi3"):
        p = os.path.join(d, f"{arch}.gguf")
        write_gguf_model(p, cfg, random_full_weights(cfg, torch.device("cpu"), seed=4, std=0.1), arch=arch)
        c, m, _ = load_gguf_model(p, "cpu")
        outs.append(_greedy(c, m, list(range(9, 50))))
    assert outs[0] == outs[1]


def test_mistral_window_and_refusals():
    c = ModelConfig.from_hf_config({"model_type": "mistral", "hidden_size": 256, "num_attention_heads": 4,
                                    "max_position_embeddings": 32768, "sliding_window": 4096})
    assert c.arch == "llama" and c.max_position == 4096
    c = ModelConfig.from_hf_config({"model_type": "mistral", "hidden_size": 256, "num_attention_heads": 4,
                                    "max_position_embeddings": 32768, "sliding_window": None})
    assert c.max_position == 32768
    with pytest.raises(ValueError, match="model_type 'falcon' is not supported"):
        ModelConfig.from_hf_config({"model_type": "falcon"})
    with pytest.raises(ValueError, match="partial rotary"):
        ModelConfig.from_hf_config({"model_type": "phi3", "partial_rotary_factor": 0.5})


def test_unsupported_gguf_architecture_is_refused():
    import numpy as np
    from gguf import GGUFReader, GGUFWriter

    from kapsl_sdk_b200.loaders.gguf import gguf_config

    p = os.path.join(tempfile.mkdtemp(), "g.gguf")
    w = GGUFWriter(p, "falcon")
    w.add_block_count(1)
    w.add_tensor("token_embd.weight", np.zeros((4, 4), np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(ValueError, match="GGUF architecture 'falcon' is not supported"):
        gguf_config(GGUFReader(p))


def qwen3_tiny():
    return ModelConfig(name="q3", arch="qwen3", vocab_size=300, hidden_size=64, intermediate_size=128, num_layers=2,
                       num_heads=4, num_kv_heads=2, head_dim=16, max_position=256, bos_token_id=None,
                       eos_token_id=None, qk_norm=True)


def test_qwen3_qk_norm_cpu_matches_oracle_and_round_trips():
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.loaders.gguf import load_gguf_model, write_gguf_model
    from kapsl_sdk_b200.loaders.hf import load_hf_model, save_hf_model
    from kapsl_sdk_b200.models.llama import random_full_weights, reference_forward

    cfg = qwen3_tiny()
    prompt = list(range(11, 70))
    ecfg = EngineConfig(max_num_seqs=2, max_num_batched_tokens=64, max_model_len=200, num_blocks=32)
    eng = LLMEngine(cfg, device="cpu", engine_cfg=ecfg, seed=0)
    out = eng.generate([prompt], SamplingParams.greedy(6, ignore_eos=True))[0]
    m = eng.model
    assert all("q_norm" in L for L in m.layers)
    toks = list(prompt)
    for _ in range(6):
        toks.append(int(reference_forward(cfg, m.layers, m.embed, m.lm_head, m.final_norm, toks)[-1].argmax()))
    assert out == toks[len(prompt):]
    # the norms change the result (they are not ones)
    plain = ModelConfig(**{**cfg.to_dict(), "qk_norm": False, "arch": "qwen2"})
    no_norm = [{k: v for k, v in L.items() if k not in ("q_norm", "k_norm")} for L in m.layers]
    assert not torch.allclose(reference_forward(cfg, m.layers, m.embed, m.lm_head, m.final_norm, prompt),
                              reference_forward(plain, no_norm, m.embed, m.lm_head, m.final_norm, prompt))
    d = tempfile.mkdtemp()
    save_hf_model(os.path.join(d, "hf"), cfg, random_full_weights(cfg, torch.device("cpu"), seed=5, std=0.1))
    c_hf, m_hf, _ = load_hf_model(os.path.join(d, "hf"), "cpu")
    assert c_hf.qk_norm and c_hf.arch == "qwen3"
    p = os.path.join(d, "q3.gguf")
    write_gguf_model(p, cfg, random_full_weights(cfg, torch.device("cpu"), seed=5, std=0.1), arch="qwen3")
    c_g, m_g, _ = load_gguf_model(p, "cpu")
    assert c_g.qk_norm
    assert _greedy(c_hf, m_hf, prompt) == _greedy(c_g, m_g, prompt)


def test_qwen3_is_refused_on_the_gpu_path():
    from kapsl_sdk_b200.llm.engine import LLMEngine

    with pytest.raises(ValueError, match="CPU backend only"):
        LLMEngine(qwen3_tiny(), device="cuda")
