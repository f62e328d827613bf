"""GGUF Q4_K weights kept quantized on the CPU backend: the C++ kernel and the
row-block path match a dense matmul with the dequantized weights, and an
engine on a Q4_K GGUF serves the same tokens quantized as dequantized; the
int8-activation decode kernel matches its integer statement."""
import os

import numpy as np
import pytest
import torch

from kapsl_sdk_b200.loaders.gguf import dequant_q4_k, quantize_q4_k
from kapsl_sdk_b200.quantization import Q4KRows


@pytest.mark.parametrize("T", [1, 5, 16, 17, 40])
def test_q4k_rows_matmul_matches_dequantized(T):
    rng = np.random.default_rng(T)
    N, K = 96, 512
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.1
    raw = quantize_q4_k(w.reshape(-1)).reshape(N, -1)
    q = Q4KRows(raw, K)
    dense = torch.from_numpy(dequant_q4_k(raw.reshape(-1)).reshape(N, K))
    assert torch.equal(q.dequantize(), dense)
    x = torch.from_numpy(rng.standard_normal((T, K)).astype(np.float32))
    ref = x @ dense.T
    torch.testing.assert_close(q.matmul(x, row_block=32, int8=False), ref, rtol=1e-4, atol=1e-4)
    # int8 activations (decode sizes): within the rounding of x to 8 bits per 256-value block
    got = q.matmul(x, row_block=32, int8=True)
    assert (got - ref).abs().max() <= 0.02 * ref.abs().max()
    if T <= 16:  # and exactly the integer statement of the same arithmetic
        xb = x.reshape(T, K // 256, 256)
        dx = xb.abs().amax(-1, keepdim=True) / 127
        xq = torch.where(dx > 0, torch.round(xb / dx).clamp(-127, 127), torch.zeros_like(xb))
        torch.testing.assert_close(got, (xq * dx).reshape(T, K) @ dense.T, rtol=2e-4, atol=2e-4)
    sub = q.take(np.array([5, 1, 7])).rows(1, 3)
    assert torch.equal(sub.dequantize(), dense[[1, 7]])


def test_engine_on_q4k_gguf_keeps_weights_quantized(tmp_path, monkeypatch):
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.loaders.gguf import load_gguf_model, write_gguf_model
    from kapsl_sdk_b200.models.config import ModelConfig
    from kapsl_sdk_b200.models.llama import random_full_weights

    cfg = ModelConfig(name="q", arch="llama", vocab_size=300, hidden_size=256, intermediate_size=512, num_layers=2,
                      num_heads=4, num_kv_heads=2, head_dim=64, max_position=256, bos_token_id=None,
                      eos_token_id=None)
    p = str(tmp_path / "m.gguf")
    write_gguf_model(p, cfg, random_full_weights(cfg, torch.device("cpu"), seed=1, std=0.05), quant="q4_k")
    c_q, m_q, _ = load_gguf_model(p, "cpu")
    assert isinstance(m_q.layers[0]["qkv"], Q4KRows) and isinstance(m_q.layers[0]["down"], Q4KRows)
    monkeypatch.setenv("KAPSL_CPU_Q4K", "0")
    c_d, m_d, _ = load_gguf_model(p, "cpu")
    assert isinstance(m_d.layers[0]["qkv"], torch.Tensor)
    torch.testing.assert_close(m_q.layers[0]["qkv"].dequantize(), m_d.layers[0]["qkv"])
    prompt = list(range(11, 60))
    monkeypatch.setenv("KAPSL_CPU_Q4K_INT8", "0")  # the fp32-activation kernel: same tokens as dense fp32
    outs = []
    for c, m in ((c_q, m_q), (c_d, m_d)):
        eng = LLMEngine(c, weights=m, device="cpu", engine_cfg=EngineConfig(
            max_num_seqs=2, max_num_batched_tokens=32, max_model_len=128, num_blocks=32), seed=0)
        outs.append(eng.generate([prompt], SamplingParams.greedy(8, ignore_eos=True))[0])
    assert outs[0] == outs[1]


def test_q6k_rows_and_mixed_stack_match_dequantized():
    from gguf import GGMLQuantizationType as Q
    from gguf import quants

    from kapsl_sdk_b200.loaders.gguf import quantize_q6_k
    from kapsl_sdk_b200.models.cpu_model import _cat_rows
    from kapsl_sdk_b200.quantization import Q6KRows, RowStack

    rng = np.random.default_rng(3)
    N, K = 80, 512
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.05
    raw = quantize_q6_k(w.reshape(-1)).reshape(N, -1)
    dense = torch.from_numpy(quants.dequantize(raw.reshape(-1, 210), Q.Q6_K).reshape(N, K).copy())
    assert (dense - torch.from_numpy(w)).abs().max() <= 0.02 * abs(w).max()  # 6-bit codes of the input
    q6 = Q6KRows(raw, K)
    assert torch.equal(q6.dequantize(), dense)
    q4 = Q4KRows(quantize_q4_k(w.reshape(-1)).reshape(N, -1), K)
    both = _cat_rows([q4, q6, torch.from_numpy(w[:8])])  # Q4_K + Q6_K + fp32 rows
    assert isinstance(both, RowStack) and both.shape == (2 * N + 8, K)
    full = torch.cat([q4.dequantize(), dense, torch.from_numpy(w[:8])])
    torch.testing.assert_close(both.dequantize(), full)
    for T in (1, 9, 16, 40):
        x = torch.from_numpy(rng.standard_normal((T, K)).astype(np.float32))
        ref = x @ full.T
        assert (both.matmul(x) - ref).abs().max() <= 0.02 * ref.abs().max()
        if T <= 16:  # Q6_K int8 kernel = its integer statement
            xb = x.reshape(T, K // 256, 256)
            dx = xb.abs().amax(-1, keepdim=True) / 127
            xq = torch.where(dx > 0, torch.round(xb / dx).clamp(-127, 127), torch.zeros_like(xb))
            torch.testing.assert_close(q6.matmul(x), (xq * dx).reshape(T, K) @ dense.T, rtol=2e-4, atol=2e-4)


def test_engine_on_q4_k_m_mix(tmp_path):
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.loaders.gguf import load_gguf_model, write_gguf_model
    from kapsl_sdk_b200.models.config import ModelConfig
    from kapsl_sdk_b200.models.llama import random_full_weights
    from kapsl_sdk_b200.quantization import Q6KRows, RowStack

    cfg = ModelConfig(name="q", arch="llama", vocab_size=256, hidden_size=256, intermediate_size=512, num_layers=2,
                      num_heads=4, num_kv_heads=2, head_dim=64, max_position=256, bos_token_id=None,
                      eos_token_id=None)
    p = str(tmp_path / "m.gguf")
    write_gguf_model(p, cfg, random_full_weights(cfg, torch.device("cpu"), seed=2, std=0.05), quant="q4_k_m")
    c, m, _ = load_gguf_model(p, "cpu")
    assert isinstance(m.layers[0]["qkv"], RowStack) and isinstance(m.layers[0]["down"], Q6KRows)
    assert isinstance(m.lm_head, Q6KRows)
    eng = LLMEngine(c, weights=m, device="cpu", engine_cfg=EngineConfig(max_num_seqs=2, max_num_batched_tokens=32,
                                                                       max_model_len=128, num_blocks=32), seed=0)
    out = eng.generate([list(range(11, 50))], SamplingParams.greedy(6, ignore_eos=True))[0]
    assert len(out) == 6


def test_q80_rows_match_gguf_and_integer_statement(tmp_path):
    from gguf import GGMLQuantizationType as Q
    from gguf import quants

    from kapsl_sdk_b200.quantization import Q80Rows

    rng = np.random.default_rng(4)
    N, K = 40, 768
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.05
    raw = quants.quantize(w, Q.Q8_0)
    dense = torch.from_numpy(quants.dequantize(raw, Q.Q8_0).reshape(N, K).copy())
    q8 = Q80Rows(raw, K)
    assert torch.equal(q8.dequantize(), dense)
    for T in (1, 16, 30):
        x = torch.from_numpy(rng.standard_normal((T, K)).astype(np.float32))
        ref = x @ dense.T
        got = q8.matmul(x)
        assert (got - ref).abs().max() <= 0.02 * ref.abs().max()
        if T <= 16:
            xb = x.reshape(T, K // 256, 256)
            dx = xb.abs().amax(-1, keepdim=True) / 127
            xq = torch.where(dx > 0, torch.round(xb / dx).clamp(-127, 127), torch.zeros_like(xb))
            torch.testing.assert_close(got, (xq * dx).reshape(T, K) @ dense.T, rtol=2e-4, atol=2e-4)


def test_engine_on_q8_0_gguf(tmp_path):
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.loaders.gguf import load_gguf_model, write_gguf_model
    from kapsl_sdk_b200.models.config import ModelConfig
    from kapsl_sdk_b200.models.llama import random_full_weights
    from kapsl_sdk_b200.quantization import Q80Rows

    cfg = ModelConfig(name="q", arch="llama", vocab_size=256, hidden_size=256, intermediate_size=512, num_layers=2,
                      num_heads=4, num_kv_heads=2, head_dim=64, max_position=256, bos_token_id=None,
                      eos_token_id=None)
    p = str(tmp_path / "m.gguf")
    write_gguf_model(p, cfg, random_full_weights(cfg, torch.device("cpu"), seed=2, std=0.05), quant="q8_0")
    c, m, _ = load_gguf_model(p, "cpu")
    assert isinstance(m.layers[0]["qkv"], Q80Rows) and isinstance(m.layers[1]["gate_up"], Q80Rows)
    eng = LLMEngine(c, weights=m, device="cpu", engine_cfg=EngineConfig(max_num_seqs=2, max_num_batched_tokens=32,
                                                                       max_model_len=128, num_blocks=32), seed=0)
    assert len(eng.generate([list(range(11, 50))], SamplingParams.greedy(6, ignore_eos=True))[0]) == 6
