"""LLM serving of a decoder export through the ONNX interpreter: a small
GenAI-style graph (embedding Gather, SimplifiedLayerNormalization, MatMulNBits
projections, GroupQueryAttention with rotary and past KV, SiLU MLP, logits) built
here; generation with the KV cache fed back equals generation that recomputes the
whole sequence each step, the runtime loader routes such exports to this engine,
and LLMBackend serves it."""
import json
import os
import tempfile

import numpy as np
import pytest
import torch

from kapsl_sdk_b200.llm.onnx_decoder import OnnxDecoderEngine, inspect_decoder
from kapsl_sdk_b200.llm.sequence import SamplingParams
from kapsl_sdk_b200.loaders.onnx import Node, OnnxGraph, encode_model, read_model

V, HID, HQ, HK, D, FF, L = 260, 32, 4, 2, 8, 48, 2  # V covers the byte tokenizer


def _pack4(w, bs=16):
    """float [N, K] -> MatMulNBits 4-bit blocks (scale per block, zero point 8)."""
    N, K = w.shape
    blocks = w.reshape(N, K // bs, bs)
    scale = np.abs(blocks).max(-1) / 7 + 1e-8
    q = np.clip(np.round(blocks / scale[..., None]) + 8, 0, 15).astype(np.uint8)
    packed = (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)
    deq = ((q.astype(np.float32) - 8) * scale[..., None]).reshape(N, K)
    return packed, scale.astype(np.float32).reshape(-1), deq


def build_decoder(path):
    rng = np.random.default_rng(0)
    inits, nodes = {}, []

    def mm(name, x, n_out, k_in):
        w = (rng.standard_normal((n_out, k_in)) * 0.3).astype(np.float32)
        packed, scale, _ = _pack4(w)
        inits[name + ".B"], inits[name + ".s"] = packed, scale
        nodes.append(Node("MatMulNBits", [x, name + ".B", name + ".s"], [name + ".y"],
                          attrs={"K": k_in, "N": n_out, "bits": 4, "block_size": 16}, domain="com.microsoft"))
        return name + ".y"

    inits["embed"] = (rng.standard_normal((V, HID)) * 0.5).astype(np.float32)
    ang = np.arange(64)[:, None] * (1.0 / 10000 ** (np.arange(D // 2) / (D // 2)))[None]
    inits["cos"], inits["sin"] = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    inits["one"] = np.array(1, np.int64)
    inits["ax1"] = np.array([1], np.int64)
    nodes += [Node("Gather", ["embed", "input_ids"], ["h0"]),
              Node("ReduceSum", ["attention_mask", "ax1"], ["ms"], attrs={"keepdims": 0}),
              Node("Sub", ["ms", "one"], ["ms1"]), Node("Cast", ["ms1"], ["seqlens_k"], attrs={"to": 6}),
              Node("Shape", ["attention_mask"], ["mshape"]),
              Node("Gather", ["mshape", "one"], ["tot64"], attrs={"axis": 0}),
              Node("Cast", ["tot64"], ["total_len"], attrs={"to": 6})]
    h = "h0"
    for i in range(L):
        inits[f"n1.{i}"] = (1 + 0.1 * rng.standard_normal(HID)).astype(np.float32)
        inits[f"n2.{i}"] = (1 + 0.1 * rng.standard_normal(HID)).astype(np.float32)
        nodes.append(Node("SimplifiedLayerNormalization", [h, f"n1.{i}"], [f"a{i}"], attrs={"epsilon": 1e-5}))
        q = mm(f"q{i}", f"a{i}", HQ * D, HID)
        k = mm(f"k{i}", f"a{i}", HK * D, HID)
        v = mm(f"v{i}", f"a{i}", HK * D, HID)
        nodes.append(Node("GroupQueryAttention", [q, k, v, f"past_key_values.{i}.key", f"past_key_values.{i}.value",
                                                  "seqlens_k", "total_len", "cos", "sin"],
                          [f"att{i}", f"present.{i}.key", f"present.{i}.value"],
                          attrs={"num_heads": HQ, "kv_num_heads": HK, "do_rotary": 1}, domain="com.microsoft"))
        o = mm(f"o{i}", f"att{i}", HID, HQ * D)
        nodes += [Node("Add", [h, o], [f"r{i}"]),
                  Node("SimplifiedLayerNormalization", [f"r{i}", f"n2.{i}"], [f"b{i}"], attrs={"epsilon": 1e-5})]
        g = mm(f"g{i}", f"b{i}", FF, HID)
        u = mm(f"u{i}", f"b{i}", FF, HID)
        nodes += [Node("Sigmoid", [g], [f"sg{i}"]), Node("Mul", [g, f"sg{i}"], [f"si{i}"]),
                  Node("Mul", [f"si{i}", u], [f"m{i}"])]
        dn = mm(f"d{i}", f"m{i}", HID, FF)
        nodes.append(Node("Add", [f"r{i}", dn], [f"h{i + 1}"]))
        h = f"h{i + 1}"
    inits["nf"] = np.ones(HID, np.float32)
    inits["lm"] = (rng.standard_normal((HID, V)) * 0.5).astype(np.float32)
    nodes += [Node("SimplifiedLayerNormalization", [h, "nf"], ["hf"], attrs={"epsilon": 1e-5}),
              Node("MatMul", ["hf", "lm"], ["logits"])]
    inputs = ["input_ids", "attention_mask"] + [f"past_key_values.{i}.{kv}" for i in range(L) for kv in ("key", "value")]
    outputs = ["logits"] + [f"present.{i}.{kv}" for i in range(L) for kv in ("key", "value")]
    with open(path, "wb") as f:
        f.write(encode_model(nodes, inputs, outputs, inits))
    with open(os.path.join(os.path.dirname(path), "genai_config.json"), "w") as f:
        json.dump({"model": {"bos_token_id": 1, "eos_token_id": 2, "vocab_size": V, "context_length": 64,
                             "decoder": {"num_key_value_heads": HK, "head_size": D, "num_hidden_layers": L}}}, f)


@pytest.fixture(scope="module")
def export_dir():
    d = tempfile.mkdtemp()
    build_decoder(os.path.join(d, "model.onnx"))
    return d


def recompute_greedy(path, prompt, n):
    g = OnnxGraph(read_model(path))
    ids = list(prompt)
    for _ in range(n):
        feeds = {"input_ids": torch.tensor([ids]), "attention_mask": torch.ones(1, len(ids), dtype=torch.int64)}
        for i in range(L):
            feeds[f"past_key_values.{i}.key"] = torch.zeros(1, HK, 0, D)
            feeds[f"past_key_values.{i}.value"] = torch.zeros(1, HK, 0, D)
        logits = g.run(feeds)["logits"][0, -1].numpy()
        ids.append(int(np.nonzero(logits == logits.max())[0][-1]))
    return ids[len(prompt):]


def test_kv_cache_generation_equals_recomputation(export_dir):
    path = os.path.join(export_dir, "model.onnx")
    io = inspect_decoder(read_model(path))
    assert io.attention_mask == "attention_mask" and len(io.past) == L
    eng = OnnxDecoderEngine(path)
    prompts = [[5, 9, 13, 4], [7, 3]]
    outs = eng.generate(prompts, SamplingParams.greedy(6, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert o == recompute_greedy(path, p, 6)
    # seeded sampling: the stream depends on (seed, sequence id), sequence ids start at 1 per engine
    sp = SamplingParams(max_new_tokens=5, temperature=0.8, seed=7, ignore_eos=True)
    a = OnnxDecoderEngine(path).generate([[5, 9]], sp)
    b = OnnxDecoderEngine(path).generate([[5, 9]], sp)
    assert a == b and len(a[0]) == 5 and eng.kv_stats()["sequences"] == 0


def test_loader_routes_unmapped_exports_and_backend_serves(export_dir):
    from kapsl_sdk_b200.engine_api import BinaryTensorPacket, InferenceRequest, RequestMetadata
    from kapsl_sdk_b200.llm.backend import LLMBackend
    from kapsl_sdk_b200.runtime.loader import build_llm_engine

    eng, tok, rc = build_llm_engine(os.path.join(export_dir, "model.onnx"), device="cpu")
    assert isinstance(eng, OnnxDecoderEngine) and eng.cfg.vocab_size == V
    be = LLMBackend(eng, tok, rc)
    try:
        req = InferenceRequest(input=BinaryTensorPacket.from_text("hi"),
                               metadata=RequestMetadata(max_new_tokens=4, temperature=0.0))
        out = be.infer(req)
        assert out.dtype.as_str() == "string"
    finally:
        be.unload()


def test_session_continuation_reuses_the_previous_turn(export_dir):
    """A second turn of a session continues after the first turn's tokens, reusing
    their KV; the tokens equal a single request over the concatenated history."""
    path = os.path.join(export_dir, "model.onnx")
    eng = OnnxDecoderEngine(path)
    g = SamplingParams.greedy(4, ignore_eos=True)
    s1 = eng.add_request("t1", [5, 9, 13], g, session_id="chat")
    while eng.has_unfinished():
        eng.step()
    s2 = eng.add_request("t2", [7, 3], g, session_id="chat")
    assert s2.cached == len(s1.prompt_ids) + len(s1.output_ids) - 1
    while eng.has_unfinished():
        eng.step()
    hist = [5, 9, 13] + s1.output_ids + [7, 3]
    assert s2.output_ids == recompute_greedy(path, hist, 4)


def test_unary_onnx_backend_fills_decoder_inputs(tmp_path):
    """Sent only input_ids, the generic ONNX backend fills attention_mask,
    position_ids and empty past caches (shapes from the declared inputs) and
    returns the logits, equal to a run with those inputs given explicitly."""
    from kapsl_sdk_b200.engine_api import BinaryTensorPacket, InferenceRequest
    from kapsl_sdk_b200.runtime.backends import OnnxBackend

    rng = np.random.default_rng(1)
    emb = rng.standard_normal((16, 8)).astype(np.float32)
    nodes = [Node("Gather", ["emb", "input_ids"], ["h"]),
             Node("Cast", ["position_ids"], ["pf"], attrs={"to": 1}), Node("Unsqueeze", ["pf", "ax"], ["p3"]),
             Node("Add", ["h", "p3"], ["hp"]),
             Node("Cast", ["attention_mask"], ["mf"], attrs={"to": 1}), Node("Unsqueeze", ["mf", "ax"], ["m3"]),
             Node("Mul", ["hp", "m3"], ["logits"]),
             Node("Concat", ["past_key_values.0.key", "kv"], ["present.0.key"], attrs={"axis": 2}),
             Node("Concat", ["past_key_values.0.value", "kv"], ["present.0.value"], attrs={"axis": 2})]
    inits = {"emb": emb, "ax": np.array([-1], np.int64), "kv": np.zeros((1, 2, 1, 4), np.float32)}
    types = {"input_ids": (7, [None, None]), "attention_mask": (7, [None, None]), "position_ids": (7, [None, None]),
             "past_key_values.0.key": (1, [None, 2, None, 4]), "past_key_values.0.value": (1, [None, 2, None, 4])}
    inputs = list(types)
    p = str(tmp_path / "m.onnx")
    open(p, "wb").write(encode_model(nodes, inputs, ["logits", "present.0.key", "present.0.value"], inits,
                                     input_types=types))
    assert read_model(p).input_types["past_key_values.0.key"] == (1, [None, 2, None, 4])
    be = OnnxBackend(device="cpu")
    be.load(p)
    ids = np.array([[3, 5, 7]], np.int64)
    out = be.infer(InferenceRequest(input=BinaryTensorPacket.from_numpy(ids))).to_numpy()
    assert np.allclose(out, emb[ids] + np.arange(3, dtype=np.float32)[None, :, None])


def test_onnx_backend_model_info_reports_declared_types(tmp_path, monkeypatch):
    from kapsl_sdk_b200.runtime.backends import OnnxBackend

    p = str(tmp_path / "m.onnx")
    open(p, "wb").write(encode_model([Node("Relu", ["x"], ["y"])], ["x"], ["y"], {},
                                     input_types={"x": (1, [None, 4])}))
    monkeypatch.setenv("KAPSL_MODEL_PEAK_CONCURRENCY", "3")
    be = OnnxBackend(device="cpu")
    be.load(p)
    info = be.model_info()
    assert info.input_shapes == [[-1, 4]] and info.input_dtypes == ["float32"]
    assert info.output_dtypes == ["unknown"] and info.framework == "onnx" and info.peak_concurrency == 3


def test_onnx_backend_rejects_duplicate_additional_inputs(tmp_path):
    from kapsl_sdk_b200.engine_api import (BinaryTensorPacket, EngineError, InferenceRequest, NamedTensor)
    from kapsl_sdk_b200.runtime.backends import OnnxBackend

    p = str(tmp_path / "m.onnx")
    open(p, "wb").write(encode_model([Node("Add", ["x", "b"], ["y"])], ["x", "b"], ["y"], {}))
    be = OnnxBackend(device="cpu")
    be.load(p)
    one = BinaryTensorPacket.from_numpy(np.ones(2, np.float32))
    req = InferenceRequest(input=one, additional_inputs=[NamedTensor("b", one), NamedTensor("b", one)])
    with pytest.raises(EngineError, match="Duplicate additional input name: b"):
        be.infer(req)
    req = InferenceRequest(input=one, additional_inputs=[NamedTensor("b", one)])
    assert np.allclose(be.infer(req).to_numpy(), 2.0)
