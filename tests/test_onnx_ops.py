"""ONNX interpreter operators beyond the core set, each run through an
encoded ModelProto (encode_model -> read_model -> OnnxGraph) and compared
with a numpy / torch statement of the operator."""
import os
import tempfile

import numpy as np
import pytest
import torch

from kapsl_sdk_b200.loaders.onnx import Node, OnnxGraph, encode_model, read_model

rng = np.random.default_rng(0)


def run(nodes, feeds: dict, outputs, inits=None):
    p = os.path.join(tempfile.mkdtemp(), "m.onnx")
    with open(p, "wb") as f:
        f.write(encode_model(nodes, list(feeds), outputs, inits or {}))
    out = OnnxGraph(read_model(p)).run(feeds)
    return [out[o].numpy() for o in outputs]


X = rng.standard_normal((2, 3, 4)).astype(np.float32)


@pytest.mark.parametrize("op,ref", [
    ("Exp", np.exp), ("Neg", np.negative), ("Abs", np.abs), ("Floor", np.floor), ("Ceil", np.ceil),
    ("Sign", np.sign), ("Sin", np.sin), ("Cos", np.cos), ("Round", np.round),
    ("Softplus", lambda x: np.log1p(np.exp(x))), ("Softsign", lambda x: x / (1 + np.abs(x))),
    ("HardSwish", lambda x: x * np.clip(x / 6 + 0.5, 0, 1)),
])
def test_unary(op, ref):
    (y,) = run([Node(op, ["x"], ["y"])], {"x": X}, ["y"])
    assert np.allclose(y, ref(X), atol=1e-5)


def test_parameterised_activations():
    (y,) = run([Node("LeakyRelu", ["x"], ["y"], attrs={"alpha": 0.1})], {"x": X}, ["y"])
    assert np.allclose(y, np.where(X > 0, X, 0.1 * X))
    (y,) = run([Node("Elu", ["x"], ["y"], attrs={"alpha": 0.5})], {"x": X}, ["y"])
    assert np.allclose(y, np.where(X > 0, X, 0.5 * (np.exp(X) - 1)), atol=1e-6)
    (y,) = run([Node("HardSigmoid", ["x"], ["y"], attrs={"alpha": 0.3, "beta": 0.4})], {"x": X}, ["y"])
    assert np.allclose(y, np.clip(0.3 * X + 0.4, 0, 1))
    (y,) = run([Node("Gelu", ["x"], ["y"], attrs={"approximate": "tanh"})], {"x": X}, ["y"])
    assert np.allclose(y, torch.nn.functional.gelu(torch.from_numpy(X), approximate="tanh").numpy(), atol=1e-6)
    lo, hi = np.array(-0.5, np.float32), np.array(0.25, np.float32)
    (y,) = run([Node("Clip", ["x", "lo", "hi"], ["y"])], {"x": X}, ["y"], {"lo": lo, "hi": hi})
    assert np.allclose(y, np.clip(X, -0.5, 0.25))
    slope = np.array([0.1, 0.2, 0.3, 0.4], np.float32)
    (y,) = run([Node("PRelu", ["x", "s"], ["y"])], {"x": X}, ["y"], {"s": slope})
    assert np.allclose(y, np.where(X >= 0, X, X * slope))


def test_variadic_compare_logic_and_where():
    a, b, c = (rng.standard_normal((3, 4)).astype(np.float32) for _ in range(3))
    ys = run([Node("Max", ["a", "b", "c"], ["mx"]), Node("Min", ["a", "b"], ["mn"]), Node("Sum", ["a", "b", "c"], ["s"]),
              Node("Mean", ["a", "b"], ["m"]), Node("Less", ["a", "b"], ["lt"]), Node("GreaterOrEqual", ["a", "b"], ["ge"]),
              Node("Where", ["lt", "a", "b"], ["w"]), Node("And", ["lt", "ge"], ["nd"]), Node("Not", ["lt"], ["nt"])],
             {"a": a, "b": b, "c": c}, ["mx", "mn", "s", "m", "w", "nd", "nt"])
    assert np.allclose(ys[0], np.maximum(np.maximum(a, b), c)) and np.allclose(ys[1], np.minimum(a, b))
    assert np.allclose(ys[2], a + b + c, atol=1e-6) and np.allclose(ys[3], (a + b) / 2)
    assert np.allclose(ys[4], np.where(a < b, a, b)) and not ys[5].any() and (ys[6] == (a >= b)).all()
    ia, ib = np.array([7, -7, 7], np.int64), np.array([3, 3, -3], np.int64)
    (m0, m1) = run([Node("Mod", ["a", "b"], ["m0"]), Node("Mod", ["a", "b"], ["m1"], attrs={"fmod": 1})],
                   {"a": ia, "b": ib}, ["m0", "m1"])
    assert m0.tolist() == [1, 2, -2] and m1.tolist() == [1, -1, 1]


def test_shape_ops():
    x = rng.standard_normal((2, 1, 3)).astype(np.float32)
    shp = np.array([2, 4, 3], np.int64)
    (y,) = run([Node("Expand", ["x", "s"], ["y"])], {"x": x}, ["y"], {"s": shp})
    assert np.allclose(y, np.broadcast_to(x, (2, 4, 3)))
    (y,) = run([Node("Tile", ["x", "r"], ["y"])], {"x": x}, ["y"], {"r": np.array([1, 2, 2], np.int64)})
    assert np.allclose(y, np.tile(x, (1, 2, 2)))
    z = rng.standard_normal((6, 5)).astype(np.float32)
    a, b = run([Node("Split", ["z", "sp"], ["a", "b"], attrs={"axis": 0})], {"z": z}, ["a", "b"],
               {"sp": np.array([2, 4], np.int64)})
    assert np.allclose(a, z[:2]) and np.allclose(b, z[2:])
    a, b, c = run([Node("Split", ["z"], ["a", "b", "c"], attrs={"axis": 1})], {"z": z}, ["a", "b", "c"])
    assert [t.shape[1] for t in (a, b, c)] == [2, 2, 1]
    pads = np.array([0, 1, 2, 0], np.int64)  # begin (axis0, axis1), end (axis0, axis1)
    (y,) = run([Node("Pad", ["z", "p", "v"], ["y"])], {"z": z}, ["y"], {"p": pads, "v": np.array(9.0, np.float32)})
    assert np.allclose(y, np.pad(z, ((0, 2), (1, 0)), constant_values=9.0))
    for mode in ("reflect", "edge"):
        (y,) = run([Node("Pad", ["z", "p"], ["y"], attrs={"mode": mode})], {"z": z}, ["y"], {"p": pads})
        assert np.allclose(y, np.pad(z, ((0, 2), (1, 0)), mode=mode))
    (y,) = run([Node("ConstantOfShape", ["s"], ["y"], attrs={"value": np.array([2.5], np.float32)})],
               {"s": np.array([2, 3], np.int64)}, ["y"])
    assert y.shape == (2, 3) and (y == 2.5).all()
    (y,) = run([Node("Range", ["a", "b", "d"], ["y"])],
               {"a": np.array(1, np.int64), "b": np.array(10, np.int64), "d": np.array(3, np.int64)}, ["y"])
    assert y.tolist() == [1, 4, 7]
    (y,) = run([Node("Trilu", ["z", "k"], ["y"], attrs={"upper": 0})], {"z": z}, ["y"], {"k": np.array(1, np.int64)})
    assert np.allclose(y, np.tril(z, 1))
    (y,) = run([Node("CumSum", ["z", "ax"], ["y"], attrs={"exclusive": 1, "reverse": 1})], {"z": z}, ["y"],
               {"ax": np.array(1, np.int64)})
    ref = np.flip(np.cumsum(np.flip(z, 1), 1), 1) - z
    assert np.allclose(y, ref, atol=1e-5)
    img = rng.standard_normal((1, 2, 3, 4)).astype(np.float32)
    (y,) = run([Node("Resize", ["x", "", "sc"], ["y"], attrs={"mode": "nearest"})], {"x": img}, ["y"],
               {"sc": np.array([1, 1, 2, 2], np.float32)})
    assert np.allclose(y, img.repeat(2, 2).repeat(2, 3))


def test_reductions_and_selection():
    axes = np.array([1], np.int64)
    ys = run([Node("ReduceSum", ["x", "ax"], ["s"], attrs={"keepdims": 0}), Node("ReduceMax", ["x"], ["mx"],
              attrs={"axes": [0, 2]}), Node("ReduceProd", ["x"], ["p"], attrs={"axes": [2], "keepdims": 0}),
              Node("ReduceL2", ["x"], ["l2"], attrs={"axes": [-1]}), Node("ArgMax", ["x"], ["am"], attrs={"axis": 2}),
              Node("ArgMin", ["x"], ["an"], attrs={"axis": 1, "keepdims": 0})],
             {"x": X}, ["s", "mx", "p", "l2", "am", "an"], {"ax": axes})
    assert np.allclose(ys[0], X.sum(1), atol=1e-6) and np.allclose(ys[1], X.max((0, 2), keepdims=True))
    assert np.allclose(ys[2], X.prod(2), atol=1e-6)
    assert np.allclose(ys[3], np.sqrt((X ** 2).sum(-1, keepdims=True)), atol=1e-6)
    assert (ys[4] == X.argmax(2)[..., None]).all() and (ys[5] == X.argmin(1)).all()
    v, i = run([Node("TopK", ["x", "k"], ["v", "i"], attrs={"axis": -1})], {"x": X}, ["v", "i"],
               {"k": np.array([2], np.int64)})
    assert np.allclose(v, -np.sort(-X, -1)[..., :2]) and (np.take_along_axis(X, i, -1) == v).all()
    (y,) = run([Node("LogSoftmax", ["x"], ["y"], attrs={"axis": 1})], {"x": X}, ["y"])
    assert np.allclose(y, torch.log_softmax(torch.from_numpy(X), 1).numpy(), atol=1e-6)


def test_layers():
    img = rng.standard_normal((2, 3, 5, 5)).astype(np.float32)
    g, b = rng.standard_normal(3).astype(np.float32), rng.standard_normal(3).astype(np.float32)
    (y,) = run([Node("InstanceNormalization", ["x", "g", "b"], ["y"], attrs={"epsilon": 1e-5})], {"x": img}, ["y"],
               {"g": g, "b": b})
    mu, var = img.mean((2, 3), keepdims=True), img.var((2, 3), keepdims=True)
    assert np.allclose(y, (img - mu) / np.sqrt(var + 1e-5) * g[:, None, None] + b[:, None, None], atol=1e-4)
    w = rng.standard_normal((3, 4, 3, 3)).astype(np.float32)
    (y,) = run([Node("ConvTranspose", ["x", "w"], ["y"], attrs={"strides": [2, 2], "pads": [1, 1, 1, 1],
                                                                "output_padding": [1, 1]})],
               {"x": img}, ["y"], {"w": w})
    ref = torch.nn.functional.conv_transpose2d(torch.from_numpy(img), torch.from_numpy(w), stride=2, padding=1,
                                               output_padding=1).numpy()
    assert y.shape == ref.shape and np.allclose(y, ref, atol=1e-5)
    (y,) = run([Node("GlobalMaxPool", ["x"], ["y"])], {"x": img}, ["y"])
    assert np.allclose(y, img.max((2, 3), keepdims=True))
    a, c = rng.standard_normal((2, 3, 4)).astype(np.float32), rng.standard_normal((2, 4, 5)).astype(np.float32)
    (y,) = run([Node("Einsum", ["a", "c"], ["y"], attrs={"equation": "bij,bjk->bik"})], {"a": a, "c": c}, ["y"])
    assert np.allclose(y, a @ c, atol=1e-5)
