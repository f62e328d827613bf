"""ONNX graph optimizer: folding, fusion and dead-code removal keep the
model's outputs and shrink the graph."""
import numpy as np
import pytest

from kapsl_sdk_b200.loaders.onnx import Node, OnnxGraph, encode_model, read_model
from kapsl_sdk_b200.optimizer import GraphOptimizer, OptimizationConfig


def _model(path):
    rng = np.random.default_rng(0)
    inits = {"w1": rng.standard_normal((8, 8)).astype(np.float32), "b0": rng.standard_normal(8).astype(np.float32),
             "b1": rng.standard_normal(8).astype(np.float32), "unused": np.ones(3, np.float32)}
    nodes = [
        Node("Add", ["b0", "b1"], ["bias"]),                  # constant subgraph -> folded
        Node("Identity", ["x"], ["x_id"]),                    # bypassed
        Node("Transpose", ["x_id"], ["xt"], attrs={"perm": [1, 0]}),
        Node("Transpose", ["xt"], ["xtt"], attrs={"perm": [1, 0]}),  # cancels the previous one
        Node("MatMul", ["xtt", "w1"], ["mm"]),
        Node("Add", ["mm", "bias"], ["y"]),
        Node("Relu", ["x"], ["dead"]),                        # feeds no output -> removed
    ]
    with open(path, "wb") as f:
        f.write(encode_model(nodes, ["x"], ["y"], inits))


def test_passes_shrink_graph_and_keep_outputs(tmp_path):
    src, dst = str(tmp_path / "m.onnx"), str(tmp_path / "o.onnx")
    _model(src)
    rep = GraphOptimizer(OptimizationConfig("O2")).optimize(src, dst)
    assert rep.original_nodes == 7 and rep.optimized_nodes == 2 and not rep.copied_unchanged
    assert rep.applied_passes == ["constant_folding", "operator_fusion", "dead_code_elimination"]
    a, b = read_model(src), read_model(dst)
    assert [n.op for n in b.nodes] == ["MatMul", "Add"] and "unused" not in b.initializers
    x = np.random.default_rng(1).standard_normal((4, 8)).astype(np.float32)
    ya = OnnxGraph(a).run({"x": x})["y"].numpy()
    yb = OnnxGraph(b).run({"x": x})["y"].numpy()
    np.testing.assert_allclose(ya, yb, rtol=1e-6, atol=1e-6)


def test_levels():
    assert GraphOptimizer(OptimizationConfig("o0")).passes == []
    with pytest.raises(ValueError, match="Invalid optimization level"):
        OptimizationConfig("O9")
