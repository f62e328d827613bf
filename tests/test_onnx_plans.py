"""Per-input-shape plans of the ONNX interpreter: values that depend only on the
initializers and the input shapes (shape arithmetic, constants, folded weight
transforms) are computed on the first run of a shape and reused; data-dependent
shapes and random ops are never reused; the plan cache is an LRU of the backend's
session-bucket size; shape values live on the host."""
import os
import tempfile

import numpy as np
import torch

from kapsl_sdk_b200.loaders.onnx import Node, OnnxGraph, encode_model, read_model


def load(nodes, inputs, outputs, inits, **kw):
    p = os.path.join(tempfile.mkdtemp(), "m.onnx")
    open(p, "wb").write(encode_model(nodes, inputs, outputs, inits))
    return OnnxGraph(read_model(p), **kw)


def flatten_graph():
    # y = Reshape(x @ W^T, [batch, -1]) with the target shape computed from Shape(x)
    w = np.random.default_rng(0).standard_normal((6, 4)).astype(np.float32)
    nodes = [Node("Transpose", ["W"], ["Wt"], attrs={"perm": [1, 0]}),
             Node("MatMul", ["x", "Wt"], ["h"]),
             Node("Shape", ["x"], ["sx"]),
             Node("Gather", ["sx", "zero"], ["b"], attrs={"axis": 0}),
             Node("Unsqueeze", ["b", "ax0"], ["b1"]),
             Node("Concat", ["b1", "minus1"], ["shp"], attrs={"axis": 0}),
             Node("Reshape", ["h", "shp"], ["y"])]
    inits = {"W": w, "zero": np.array(0, np.int64), "ax0": np.array([0], np.int64),
             "minus1": np.array([-1], np.int64)}
    return nodes, inits, w


def test_plan_reuses_shape_values_and_folded_weights():
    nodes, inits, w = flatten_graph()
    g = load(nodes, ["x"], ["y"], inits)
    rng = np.random.default_rng(1)
    for shape in [(2, 3, 4), (2, 3, 4), (5, 1, 4), (2, 3, 4)]:
        x = rng.standard_normal(shape).astype(np.float32)
        y = g.run({"x": x})["y"].numpy()
        assert np.allclose(y, (x @ w.T).reshape(shape[0], -1), atol=1e-5)
    assert g.stats["plans_built"] == 2 and g.stats["plan_hits"] == 2
    assert g.stats["nodes_skipped"] == 2 * 5  # Transpose, Shape, Gather, Unsqueeze, Concat
    assert g.consts["zero"].device.type == "cpu" and g.consts["W"].dtype == torch.float32


def test_data_dependent_shapes_and_random_ops_are_not_reused():
    nodes = [Node("NonZero", ["x"], ["nz"]), Node("Shape", ["nz"], ["s"]),
             Node("RandomUniformLike", ["x"], ["r"], attrs={"seed": 1.0}),
             Node("ReduceSum", ["r"], ["rs"], attrs={"keepdims": 0})]
    g = load(nodes, ["x"], ["s", "rs"], {})
    a = g.run({"x": np.array([1.0, 0.0, 2.0], np.float32)})["s"].tolist()
    b = g.run({"x": np.array([0.0, 0.0, 2.0], np.float32)})["s"].tolist()
    assert a == [1, 2] and b == [1, 1]


def test_plan_cache_is_bounded_lru():
    nodes, inits, w = flatten_graph()
    g = load(nodes, ["x"], ["y"], inits, plan_cache=2)
    for b in (1, 2, 3, 1):
        g.run({"x": np.ones((b, 2, 4), np.float32)})
    assert len(g._plans) == 2 and g.stats["plans_built"] == 4 and g.stats["plan_hits"] == 0
    g.run({"x": np.ones((1, 2, 4), np.float32)})
    assert g.stats["plan_hits"] == 1
    g0 = load(nodes, ["x"], ["y"], inits, plan_cache=0)
    g0.run({"x": np.ones((1, 2, 4), np.float32)})
    g0.run({"x": np.ones((1, 2, 4), np.float32)})
    assert g0.stats["plan_hits"] == 0 and not g0._plans


def test_value_shaped_ops_depend_on_static_arguments_only():
    # ConstantOfShape over a shape computed from the input's values is not static
    nodes = [Node("ReduceMax", ["x"], ["m"], attrs={"keepdims": 1}), Node("Cast", ["m"], ["mi"], attrs={"to": 7}),
             Node("ConstantOfShape", ["mi"], ["z"]), Node("Shape", ["z"], ["s"])]
    g = load(nodes, ["x"], ["s"], {})
    assert g.run({"x": np.array([3.0], np.float32)})["s"].tolist() == [3]
    assert g.run({"x": np.array([5.0], np.float32)})["s"].tolist() == [5]


def test_onnx_backend_serves_with_plans():
    from kapsl_sdk_b200.engine_api import BinaryTensorPacket, InferenceRequest
    from kapsl_sdk_b200.runtime.backends import OnnxBackend

    nodes, inits, w = flatten_graph()
    p = os.path.join(tempfile.mkdtemp(), "m.onnx")
    open(p, "wb").write(encode_model(nodes, ["x"], ["y"], inits))
    be = OnnxBackend(device="cpu", max_buckets=2)
    be.load(p)
    x = np.random.default_rng(3).standard_normal((2, 3, 4)).astype(np.float32)
    for _ in range(3):
        out = be.infer(InferenceRequest(input=BinaryTensorPacket.from_numpy(x))).to_numpy()
        assert np.allclose(out, (x @ w.T).reshape(2, -1), atol=1e-5)
    assert be.graph.stats["plans_built"] == 1 and be.graph.stats["plan_hits"] == 2


def test_malformed_files_raise_value_error(tmp_path):
    """Truncated and corrupted models end in ValueError (never another exception type or a hang)."""
    import random

    nodes, inits, _ = flatten_graph()
    good = encode_model(nodes, ["x"], ["y"], inits)
    rng = random.Random(0)
    p = tmp_path / "m.onnx"
    outcomes = {"ok": 0, "rejected": 0}
    for i in range(600):
        b = bytearray(good)
        if i % 3 == 0:
            b = b[:rng.randrange(len(b))]
        else:
            for _ in range(rng.randint(1, 3)):
                b[rng.randrange(len(b))] = rng.randrange(256)
        p.write_bytes(bytes(b))
        try:
            m = read_model(str(p))
            OnnxGraph(m)
            outcomes["ok"] += 1
        except ValueError:
            outcomes["rejected"] += 1
    assert outcomes["rejected"] > 100
