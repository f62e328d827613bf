"""GPTQ / AWQ / INT8 safetensors readers: pack known integer weights with each
format's layout, save, load, dequantize, compare."""
import json

import torch
from safetensors.torch import save_file

from kapsl_sdk_b200.quantization.safetensors_loaders import (AWQ_ORDER, QuantizationConfig, load_awq, load_gptq,
                                                             load_int8, load_quantized, read_quantization_config)


def _pack_rows(q):  # [K, N] 4-bit -> [K/8, N] int32, low nibble = first row
    K, N = q.shape
    v = q.view(K // 8, 8, N).to(torch.int64)
    out = torch.zeros(K // 8, N, dtype=torch.int64)
    for i in range(8):
        out |= v[:, i] << (4 * i)
    return out.to(torch.int32) if (out < 2**31).all() else (out - (out >= 2**31) * 2**32).to(torch.int32)


def _pack_cols(q, order=tuple(range(8))):  # [R, C] -> [R, C/8], slot s holds column order[s]
    R, C = q.shape
    v = q.view(R, C // 8, 8).to(torch.int64)
    out = torch.zeros(R, C // 8, dtype=torch.int64)
    for s, col in enumerate(order):
        out |= v[:, :, col] << (4 * s)
    out = out - (out >= 2**31).to(torch.int64) * 2**32
    return out.to(torch.int32)


def test_gptq_roundtrip(tmp_path):
    g = torch.Generator().manual_seed(0)
    K, N, G = 64, 16, 32
    q = torch.randint(0, 16, (K, N), generator=g)
    z = torch.randint(1, 15, (K // G, N), generator=g)
    s = (torch.rand(K // G, N, generator=g) * 0.1 + 0.01).half()
    save_file({"l.qweight": _pack_rows(q), "l.qzeros": _pack_cols(z - 1), "l.scales": s},
              str(tmp_path / "m.safetensors"))
    (tmp_path / "quantize_config.json").write_text(json.dumps({"bits": 4, "group_size": G, "desc_act": False,
                                                                "quant_method": "gptq"}))
    assert read_quantization_config(str(tmp_path)).quantization_method == "gptq"
    t = load_gptq(str(tmp_path))["l"]
    assert t.shape == (N, K)
    want = (s.float()[torch.arange(K) // G] * (q.float() - z.float()[torch.arange(K) // G])).T
    torch.testing.assert_close(t.dequantize(), want)
    assert set(load_quantized(str(tmp_path))) == {"l"}


def test_awq_roundtrip(tmp_path):
    g = torch.Generator().manual_seed(1)
    K, N, G = 32, 32, 16
    q = torch.randint(0, 16, (K, N), generator=g)
    z = torch.randint(0, 16, (K // G, N), generator=g)
    s = (torch.rand(K // G, N, generator=g) * 0.1).half()
    save_file({"a.qweight": _pack_cols(q, AWQ_ORDER), "a.qzeros": _pack_cols(z, AWQ_ORDER), "a.scales": s},
              str(tmp_path / "m.safetensors"))
    t = load_awq(str(tmp_path), QuantizationConfig("awq", 4, G))["a"]
    gi = torch.arange(K) // G
    torch.testing.assert_close(t.dequantize(), (s.float()[gi] * (q.float() - z.float()[gi])).T)


def test_int8(tmp_path):
    w = torch.randint(-128, 128, (8, 12), dtype=torch.int8)
    save_file({"x.weight": w, "x.scale": torch.tensor([0.05]), "x.zero_point": torch.tensor([3], dtype=torch.int32),
               "y.weight": torch.ones(2, 2)}, str(tmp_path / "m.safetensors"))
    t = load_int8(str(tmp_path))
    assert set(t) == {"x"}
    torch.testing.assert_close(t["x"].dequantize(), (w.float() - 3) * 0.05)
