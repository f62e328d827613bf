"""Model formats and packages: GGUF (quant blocks, read/write, serving on the
CPU backend), HF safetensors, ONNX (protobuf decode, interpreter, LLM
initializers) and .aimod packages with the model cache."""
import io
import json
import os
import tarfile
import tempfile

import numpy as np
import pytest
import torch

from kapsl_sdk_b200.models.config import ModelConfig
from kapsl_sdk_b200.models.llama import random_full_weights


def tiny(**kw):
    c = ModelConfig(name="tiny", arch="llama", vocab_size=320, hidden_size=256, intermediate_size=512, num_layers=2,
                    num_heads=4, num_kv_heads=2, head_dim=64, max_position=512, bos_token_id=1, eos_token_id=2)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def test_q4k_q6k_q80_match_gguf_reference():
    from gguf import GGMLQuantizationType as Q
    from gguf import quants

    from kapsl_sdk_b200.loaders import gguf as G

    rng = np.random.default_rng(0)
    x = (rng.standard_normal(256 * 16) * 0.02).astype(np.float32)
    q = G.quantize_q4_k(x)
    assert np.array_equal(G.dequant_q4_k(q), quants.dequantize(q.reshape(-1, 144), Q.Q4_K).reshape(-1))
    assert np.abs(G.dequant_q4_k(q) - x).max() < 0.1 * np.abs(x).max()
    q6 = rng.integers(0, 256, size=(16, 210), dtype=np.uint8)  # random Q6_K blocks with a small scale
    q6[:, 208:210] = np.full((16, 1), 0.001, np.float16).view(np.uint8).reshape(16, 2)
    assert np.allclose(G.dequant_q6_k(q6.reshape(-1)), quants.dequantize(q6, Q.Q6_K).reshape(-1))
    q8 = quants.quantize(x.reshape(-1, 256), Q.Q8_0)
    assert np.allclose(G.dequant_q8_0(q8.reshape(-1)), quants.dequantize(q8, Q.Q8_0).reshape(-1))


@pytest.mark.parametrize("quant", ["f32", "q4_k"])
def test_gguf_roundtrip_and_cpu_serving(quant):
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.loaders import gguf as G
    from kapsl_sdk_b200.models.cpu_model import CPUCausalLM

    cfg = tiny()
    d = tempfile.mkdtemp()
    p = os.path.join(d, "m.gguf")
    G.write_gguf_model(p, cfg, random_full_weights(cfg, torch.device("cpu"), 0), quant)
    c2, model, tok = G.load_gguf_model(p, "cpu")
    assert (c2.hidden_size, c2.num_heads, c2.num_kv_heads, c2.num_layers) == (256, 4, 2, 2)
    items = list(random_full_weights(cfg, torch.device("cpu"), 0))
    ref = CPUCausalLM(cfg, items[0][1], items[1][1], torch.ones(256), [t for k, t in items[2:]])
    tol = 0 if quant == "f32" else 0.1 * float(ref.layers[0]["q"].abs().max())
    q = model.layers[0]["q"]
    if quant == "q4_k":
        from kapsl_sdk_b200.quantization import Q4KRows
        assert isinstance(q, Q4KRows)  # Q4_K projections stay quantized on the CPU backend
        q = q.dequantize()
    assert (q - ref.layers[0]["q"]).abs().max() <= tol + 1e-7
    e = LLMEngine(c2, weights=model, device="cpu", engine_cfg=EngineConfig(max_num_seqs=2, max_model_len=128,
                                                                          num_blocks=32))
    out = e.generate([[5, 6, 7, 8]], SamplingParams.greedy(4, ignore_eos=True))[0]
    if quant == "f32":
        er = LLMEngine(cfg, weights=ref, device="cpu", engine_cfg=EngineConfig(max_num_seqs=2, max_model_len=128,
                                                                              num_blocks=32))
        assert out == er.generate([[5, 6, 7, 8]], SamplingParams.greedy(4, ignore_eos=True))[0]
    assert tok.decode(tok.encode("hello world")) == "hello world"


def test_hf_safetensors_roundtrip():
    from kapsl_sdk_b200.loaders.hf import load_hf_model, save_hf_model

    cfg = tiny(arch="qwen2", qkv_bias=True)
    d = tempfile.mkdtemp()
    save_hf_model(d, cfg, random_full_weights(cfg, torch.device("cpu"), 3))
    c2, m, _ = load_hf_model(d, "cpu")
    assert c2.arch == "qwen2" and c2.qkv_bias
    items = list(random_full_weights(cfg, torch.device("cpu"), 3))
    assert torch.equal(m.layers[1]["q_b"], items[3][1]["q_b"].float())


def test_onnx_decode_and_interpret():
    from kapsl_sdk_b200.loaders.onnx import Node, OnnxGraph, encode_model, read_model

    rng = np.random.default_rng(1)
    w1 = rng.standard_normal((8, 16)).astype(np.float32)
    b1 = rng.standard_normal(16).astype(np.float32)
    w2 = rng.standard_normal((16, 4)).astype(np.float32)
    nodes = [Node("MatMul", ["x", "w1"], ["h"]), Node("Add", ["h", "b1"], ["hb"]), Node("Relu", ["hb"], ["r"]),
             Node("Gemm", ["r", "w2"], ["y"], attrs={"alpha": 2.0}), Node("Softmax", ["y"], ["z"], attrs={"axis": 1})]
    blob = encode_model(nodes, ["x"], ["z"], {"w1": w1, "b1": b1, "w2": w2})
    d = tempfile.mkdtemp()
    p = os.path.join(d, "mlp.onnx")
    open(p, "wb").write(blob)
    m = read_model(p)
    assert m.inputs == ["x"] and m.outputs == ["z"] and set(m.initializers) == {"w1", "b1", "w2"}
    x = rng.standard_normal((3, 8)).astype(np.float32)
    out = OnnxGraph(m).run({"x": x})["z"].numpy()
    y = 2.0 * (np.maximum(x @ w1 + b1, 0) @ w2)
    exp = np.exp(y - y.max(1, keepdims=True))
    assert np.allclose(out, exp / exp.sum(1, keepdims=True), atol=1e-5)
    bad = encode_model([Node("StringNormalizer", ["x"], ["y"])], ["x"], ["y"], {})
    open(p, "wb").write(bad)
    with pytest.raises(ValueError, match="StringNormalizer"):
        OnnxGraph(read_model(p))


def test_onnx_backend_engine():
    from kapsl_sdk_b200.engine_api import BinaryTensorPacket, InferenceRequest
    from kapsl_sdk_b200.loaders.onnx import Node, encode_model
    from kapsl_sdk_b200.runtime.backends import OnnxBackend

    w = np.eye(4, dtype=np.float32) * 3
    p = os.path.join(tempfile.mkdtemp(), "lin.onnx")
    open(p, "wb").write(encode_model([Node("MatMul", ["x", "w"], ["y"])], ["x"], ["y"], {"w": w}))
    b = OnnxBackend(device="cpu")
    b.load(p)
    out = b.infer(InferenceRequest(BinaryTensorPacket.from_numpy(np.ones((2, 4), np.float32))))
    assert out.shape == [2, 4] and np.allclose(out.to_numpy(), 3.0)
    assert b.model_info().input_names == ["x"]


def _aimod(d, files: dict, manifest: dict) -> str:
    p = os.path.join(d, "pkg.aimod")
    with tarfile.open(p, "w:gz") as tf:
        for name, data in list(files.items()) + [("metadata.json", json.dumps(manifest).encode())]:
            ti = tarfile.TarInfo(name)
            ti.size = len(data)
            tf.addfile(ti, io.BytesIO(data))
    return p


def test_package_loader_cache_and_safety():
    from kapsl_sdk_b200.runtime.loader import PackageLoader

    d = tempfile.mkdtemp()
    man = {"project_name": "p", "framework": "onnx", "version": "2", "model_file": "m.onnx", "created_at": "now",
           "metadata": {"llm": {"max_seq_len": 64}}}
    pkg = _aimod(d, {"m.onnx": b"x"}, man)
    loader = PackageLoader(cache_dir=os.path.join(d, "cache"), max_bytes=10_000_000)
    a = loader.load(pkg)
    b = loader.load(pkg)
    assert a.root == b.root and os.path.isfile(a.model_path) and a.manifest.version == "2"
    evil = os.path.join(d, "evil.aimod")
    with tarfile.open(evil, "w:gz") as tf:
        ti = tarfile.TarInfo("../../escape.txt")
        ti.size = 1
        tf.addfile(ti, io.BytesIO(b"!"))
    with pytest.raises(ValueError, match="unsafe"):
        loader.load(evil)
    small = PackageLoader(cache_dir=os.path.join(d, "cache"), max_bytes=1)
    assert small.evict() >= 1


def test_gguf_package_serves_through_backend():
    from kapsl_sdk_b200.engine_api import BinaryTensorPacket, InferenceRequest, TensorDtype
    from kapsl_sdk_b200.llm.backend import LLMBackend
    from kapsl_sdk_b200.loaders import gguf as G
    from kapsl_sdk_b200.runtime.loader import PackageLoader, build_llm_engine

    cfg = tiny()
    d = tempfile.mkdtemp()
    g = os.path.join(d, "m.gguf")
    G.write_gguf_model(g, cfg, random_full_weights(cfg, torch.device("cpu"), 0), "f32")
    man = {"project_name": "tiny", "framework": "gguf", "version": "1", "model_file": "m.gguf",
           "metadata": {"llm": {"max_seq_len": 128, "scheduler": {"max_num_seqs": 2}, "kv_cache": {"total_blocks": 32}}},
           "hardware_requirements": {"preferred_provider": "cpu"}}
    pkg = _aimod(d, {"m.gguf": open(g, "rb").read()}, man)
    os.environ["KAPSL_MODEL_CACHE_DIR"] = os.path.join(d, "cache")
    try:
        eng, tok, rc = build_llm_engine(pkg)
    finally:
        del os.environ["KAPSL_MODEL_CACHE_DIR"]
    assert rc.sampling.temperature == 0.0 and not rc.use_chat_template
    be = LLMBackend(eng, tok, rc)
    try:
        req = InferenceRequest(BinaryTensorPacket([1, 5], TensorDtype.UTF8, b"hello"))
        req.metadata = None
        from kapsl_sdk_b200.engine_api import RequestMetadata

        req.metadata = RequestMetadata(max_new_tokens=4)
        out = be.infer(req)
        assert out.dtype is TensorDtype.UTF8
    finally:
        be.unload()
