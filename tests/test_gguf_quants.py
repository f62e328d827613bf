"""GGML block formats beyond Q4_K / Q6_K / Q8_0: this loader's dequantizers match
the gguf package's on random blocks, and models written in the legacy formats
load and generate the same greedy tokens as their dequantized weights."""
import os
import tempfile

import numpy as np
import pytest
import torch

from kapsl_sdk_b200.loaders import gguf as G

gguf = pytest.importorskip("gguf")
Q = gguf.GGMLQuantizationType

# block bytes and the byte offsets of f16 fields (scales) for each format
FORMATS = {
    "Q4_0": (18, [0], G.dequant_q4_0), "Q4_1": (20, [0, 2], G.dequant_q4_1),
    "Q5_0": (22, [0], G.dequant_q5_0), "Q5_1": (24, [0, 2], G.dequant_q5_1),
    "Q2_K": (84, [80, 82], G.dequant_q2_k), "Q3_K": (110, [108], G.dequant_q3_k),
    "Q5_K": (176, [0, 2], G.dequant_q5_k),
}


@pytest.mark.parametrize("name", sorted(FORMATS))
def test_dequantizers_match_the_gguf_package(name):
    nb, f16_at, fn = FORMATS[name]
    rng = np.random.default_rng(len(name) * 7 + nb)
    b = rng.integers(0, 256, (96, nb), dtype=np.uint8)
    for p in f16_at:  # finite scales: random bytes can spell inf / nan halves
        b[:, p:p + 2] = np.frombuffer(rng.uniform(-0.2, 0.2, 96).astype(np.float16).tobytes(),
                                      np.uint8).reshape(96, 2)
    want = gguf.quants.dequantize(b, getattr(Q, name)).reshape(-1)
    got = fn(b)
    assert got.dtype == np.float32 and np.array_equal(got, want)


@pytest.mark.parametrize("quant", ["q4_0", "q5_1"])
def test_legacy_quant_model_loads_and_generates(quant):
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.config import ModelConfig
    from kapsl_sdk_b200.models.llama import random_full_weights

    cfg = ModelConfig(name="t", arch="llama", vocab_size=512, hidden_size=256, intermediate_size=512, num_layers=2,
                      num_heads=4, num_kv_heads=2, head_dim=64, max_position=256, bos_token_id=1, eos_token_id=2)
    d = tempfile.mkdtemp()
    path = os.path.join(d, f"m-{quant}.gguf")
    G.write_gguf_model(path, cfg, random_full_weights(cfg, torch.device("cpu"), seed=3, std=0.05), quant=quant)
    reader = gguf.GGUFReader(path)
    assert getattr(Q, quant.upper()) in {t.tensor_type for t in reader.tensors}
    c2, model, _ = G.load_gguf_model(path, "cpu")
    # the loaded weights are exactly the file's blocks dequantized
    t = next(t for t in reader.tensors if t.name == "blk.0.ffn_down.weight")
    ref = gguf.quants.dequantize(np.asarray(t.data), t.tensor_type).reshape(cfg.hidden_size, -1)
    assert np.array_equal(model.layers[0]["down"].numpy(), ref)
    eng = LLMEngine(c2, weights=model, device="cpu", engine_cfg=EngineConfig(max_num_seqs=2, max_model_len=128,
                                                                             num_blocks=32))
    out = eng.generate([[5, 6, 7, 8, 9]], SamplingParams.greedy(6, ignore_eos=True))[0]
    assert len(out) == 6 and all(0 <= x < cfg.vocab_size for x in out)
