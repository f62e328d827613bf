"""HAL kernel traits on the CPU backend against the reference ops; model paths."""
import os

import torch

from kapsl_sdk_b200.hal.kernels import AttentionConfig, TensorView, create_backend
from kapsl_sdk_b200.llm.model_paths import find_model_asset, find_model_root
from kapsl_sdk_b200.ops import reference as ref


def test_cpu_backend_attention_and_swiglu():
    be = create_backend("cpu")
    g = torch.Generator().manual_seed(0)
    q, k, v = torch.randn(2, 4, 5, 16, generator=g), torch.randn(2, 2, 9, 16, generator=g), torch.randn(2, 2, 9, 16, generator=g)
    out = be.attention(q, k, v)
    for b in range(2):
        want = ref.attention(q[b].permute(1, 0, 2), k[b].permute(1, 0, 2), v[b].permute(1, 0, 2), 16 ** -0.5, 4)
        torch.testing.assert_close(out[b].permute(1, 0, 2), want, atol=1e-5, rtol=1e-4)
    full = be.attention(q, k, v, AttentionConfig(causal=False))
    assert full.shape == q.shape
    gt, up = torch.randn(3, 7, generator=g), torch.randn(3, 7, generator=g)
    torch.testing.assert_close(be.fused_swiglu(gt, up), gt * torch.sigmoid(gt) * up, atol=1e-6, rtol=1e-5)
    assert TensorView(list(range(6)), (2, 3)).as_tensor().shape == (2, 3)


def test_model_paths(tmp_path):
    (tmp_path / "m" / "onnx-export").mkdir(parents=True)
    (tmp_path / "m" / "metadata.json").write_text("{}")
    (tmp_path / "m" / "onnx-export" / "model.onnx").write_bytes(b"")
    assert find_model_root(str(tmp_path / "m" / "onnx-export" / "model.onnx")) == str(tmp_path / "m")
    assert find_model_asset(str(tmp_path / "m"), "model.onnx").endswith(os.path.join("onnx-export", "model.onnx"))
    assert find_model_root(str(tmp_path)) is None
