"""The ONNX interpreter on the GPU: shape arithmetic stays on the host (small
integer tensors), data on the device, and results equal the CPU run; repeated
shapes reuse their plan."""
import os
import tempfile

import numpy as np
import pytest
import torch

from kapsl_sdk_b200.loaders.onnx import Node, OnnxGraph, OnnxModel, encode_model, read_model

pytestmark = pytest.mark.gpu


def test_interpreter_on_cuda_matches_cpu():
    rng = np.random.default_rng(0)
    B, S, H, D = 2, 5, 2, 8
    wq = (rng.standard_normal((H * D, H * D)) * 0.2).astype(np.float32)
    body = OnnxModel([Node("Add", ["acc", "one"], ["acc_out"]), Node("Identity", ["c"], ["c_out"])],
                     ["i", "c", "acc"], ["c_out", "acc_out"], {})
    nodes = [Node("MatMul", ["x", "Wq"], ["q"]),
             Node("Shape", ["x"], ["sx"]), Node("Gather", ["sx", "zero"], ["b"], attrs={"axis": 0}),
             Node("Gather", ["sx", "one_i"], ["s"], attrs={"axis": 0}),
             Node("Unsqueeze", ["b", "ax0"], ["b1"]), Node("Unsqueeze", ["s", "ax0"], ["s1"]),
             Node("Concat", ["b1", "s1", "heads", "hd"], ["shp"], attrs={"axis": 0}),
             Node("Reshape", ["q", "shp"], ["q4"]), Node("Transpose", ["q4"], ["qh"], attrs={"perm": [0, 2, 1, 3]}),
             Node("Attention", ["qh", "qh", "qh"], ["att"], attrs={"is_causal": 1}),
             Node("Loop", ["trip", "", "att"], ["y"], attrs={"body": body})]
    inits = {"Wq": wq, "zero": np.array(0, np.int64), "one_i": np.array(1, np.int64), "ax0": np.array([0], np.int64),
             "heads": np.array([H], np.int64), "hd": np.array([D], np.int64), "trip": np.array(3, np.int64),
             "one": np.array(1.0, np.float32)}
    p = os.path.join(tempfile.mkdtemp(), "m.onnx")
    open(p, "wb").write(encode_model(nodes, ["x"], ["y"], inits))
    m = read_model(p)
    x = rng.standard_normal((B, S, H * D)).astype(np.float32)
    ref = OnnxGraph(m, "cpu").run({"x": x})["y"]
    g = OnnxGraph(m, "cuda:0")
    assert g.consts["zero"].device.type == "cpu" and g.consts["Wq"].is_cuda
    for _ in range(3):
        out = g.run({"x": x})["y"]
        assert out.is_cuda
        torch.testing.assert_close(out.cpu(), ref, atol=1e-4, rtol=1e-4)
    assert g.stats["plan_hits"] == 2
