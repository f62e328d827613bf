"""ONNX interpreter operators beyond the core set, each a one-node graph encoded,
decoded and run by ``OnnxGraph`` against a NumPy statement of the ONNX spec."""
import os
import tempfile

import numpy as np
import pytest

from kapsl_sdk_b200.loaders.onnx import Node, OnnxGraph, encode_model, read_model

rng = np.random.default_rng(4)


def run1(op, feeds: dict, attrs=None, inits=None, n_out=1):
    ins = list(feeds) + list(inits or {})
    outs = [f"y{i}" for i in range(n_out)]
    blob = encode_model([Node(op, ins, outs, attrs=attrs or {})], list(feeds), outs, inits or {})
    p = os.path.join(tempfile.mkdtemp(), "m.onnx")
    open(p, "wb").write(blob)
    res = OnnxGraph(read_model(p)).run(feeds)
    return [res[o].numpy() for o in outs] if n_out > 1 else res[outs[0]].numpy()


def test_gather_scatter_elements():
    x = rng.standard_normal((3, 4)).astype(np.float32)
    idx = np.array([[0, -1, 2, 1], [3, 0, 0, 2]], np.int64)
    want = np.take_along_axis(x[:2], np.where(idx < 0, idx + 4, idx), axis=1)
    assert np.allclose(run1("GatherElements", {"x": x}, {"axis": 1}, {"i": idx}), want)
    data = np.zeros((3, 3), np.float32)
    ind = np.array([[1, 0, 2], [0, 2, 1]], np.int64)
    upd = np.array([[1.0, 1.1, 1.2], [2.0, 2.1, 2.2]], np.float32)
    want = data.copy()
    for i in range(2):
        for j in range(3):
            want[ind[i, j], j] = upd[i, j]
    assert np.allclose(run1("ScatterElements", {"d": data}, {"axis": 0}, {"i": ind, "u": upd}), want)
    want_add = np.ones((3, 3), np.float32)
    for i in range(2):
        for j in range(3):
            want_add[ind[i, j], j] += upd[i, j]
    got = run1("ScatterElements", {"d": np.ones((3, 3), np.float32)}, {"axis": 0, "reduction": "add"},
               {"i": ind, "u": upd})
    assert np.allclose(got, want_add)


def test_scatter_nd_gather_nd():
    data = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    idx = np.array([[0, 1], [1, 2]], np.int64)
    upd = -np.ones((2, 4), np.float32)
    want = data.copy()
    want[0, 1] = -1
    want[1, 2] = -1
    assert np.allclose(run1("ScatterND", {"d": data}, {}, {"i": idx, "u": upd}), want)
    assert np.allclose(run1("GatherND", {"d": data}, {}, {"i": idx}), np.stack([data[0, 1], data[1, 2]]))


def test_one_hot_and_nonzero():
    ind = np.array([0, 2, -1, 5], np.int64)
    got = run1("OneHot", {"i": ind}, {}, {"d": np.array([3], np.int64), "v": np.array([-1.0, 4.0], np.float32)})
    want = np.full((4, 3), -1.0, np.float32)
    want[0, 0] = want[1, 2] = want[2, 2] = 4.0  # -1 counts from the end; 5 is out of range
    assert np.allclose(got, want)
    x = np.array([[1, 0], [0, 3]], np.float32)
    assert np.array_equal(run1("NonZero", {"x": x}), np.array(np.nonzero(x)))


@pytest.mark.parametrize("mode", ["DCR", "CRD"])
def test_depth_space(mode):
    x = rng.standard_normal((1, 8, 2, 3)).astype(np.float32)
    b = 2
    N, C, H, W = x.shape
    if mode == "DCR":
        want = x.reshape(N, b, b, C // 4, H, W).transpose(0, 3, 4, 1, 5, 2).reshape(N, C // 4, H * b, W * b)
    else:
        want = x.reshape(N, C // 4, b, b, H, W).transpose(0, 1, 4, 2, 5, 3).reshape(N, C // 4, H * b, W * b)
    got = run1("DepthToSpace", {"x": x}, {"blocksize": 2, "mode": mode})
    assert np.allclose(got, want)
    if mode == "DCR":  # SpaceToDepth inverts the DCR layout
        assert np.allclose(run1("SpaceToDepth", {"x": got}, {"blocksize": 2}), x)


def test_quantize_dequantize():
    x = np.array([-1.0, 0.0, 0.25, 1.5, 300.0], np.float32)
    s, z = np.array(0.5, np.float32), np.array(10, np.uint8)
    q = run1("QuantizeLinear", {"x": x}, {}, {"s": s, "z": z})
    assert q.dtype == np.uint8 and q.tolist() == [8, 10, 10, 13, 255]  # 0.25 / 0.5 = 0.5 rounds to even
    assert np.allclose(run1("DequantizeLinear", {"q": q}, {}, {"s": s, "z": z}), (q.astype(np.float32) - 10) * 0.5)
    x2 = rng.standard_normal((2, 3)).astype(np.float32)
    sc = np.array([0.1, 0.2, 0.05], np.float32)
    zp = np.array([0, -3, 5], np.int8)
    q2 = run1("QuantizeLinear", {"x": x2}, {"axis": 1}, {"s": sc, "z": zp})
    assert q2.dtype == np.int8
    assert np.array_equal(q2, np.clip(np.round(x2 / sc) + zp, -128, 127).astype(np.int8))


def test_norms_and_reductions():
    x = rng.standard_normal((2, 6, 4)).astype(np.float32)
    g = 3
    xr = x.reshape(2, g, -1)
    norm = ((xr - xr.mean(-1, keepdims=True)) / np.sqrt(xr.var(-1, keepdims=True) + 1e-5)).reshape(x.shape)
    sc, bi = rng.standard_normal(6).astype(np.float32), rng.standard_normal(6).astype(np.float32)
    got = run1("GroupNormalization", {"x": x}, {"num_groups": g}, {"s": sc, "b": bi})
    assert np.allclose(got, norm * sc[None, :, None] + bi[None, :, None], atol=1e-4)
    assert np.allclose(run1("LpNormalization", {"x": x}, {"axis": -1, "p": 2}),
                       x / np.linalg.norm(x, axis=-1, keepdims=True), atol=1e-5)
    axes = np.array([1], np.int64)
    assert np.allclose(run1("ReduceLogSumExp", {"x": x}, {"keepdims": 0}, {"a": axes}),
                       np.log(np.exp(x).sum(1)), atol=1e-5)
    assert np.allclose(run1("ReduceSumSquare", {"x": x}, {}, {"a": axes}), (x * x).sum(1, keepdims=True), atol=1e-5)
    assert np.allclose(run1("ReduceL1", {"x": x}, {}, {"a": axes}), np.abs(x).sum(1, keepdims=True), atol=1e-5)


def test_activations_and_selection():
    x = np.linspace(-3, 3, 13, dtype=np.float32)
    assert np.allclose(run1("Mish", {"x": x}), x * np.tanh(np.log1p(np.exp(x))), atol=1e-6)
    assert np.allclose(run1("Celu", {"x": x}, {"alpha": 2.0}),
                       np.maximum(0, x) + np.minimum(0, 2.0 * (np.exp(x / 2.0) - 1)), atol=1e-6)
    assert np.allclose(run1("ThresholdedRelu", {"x": x}, {"alpha": 1.0}), np.where(x > 1.0, x, 0))
    assert np.allclose(run1("Shrink", {"x": x}, {"lambd": 1.0, "bias": 0.5}),
                       np.where(x < -1, x + 0.5, np.where(x > 1, x - 0.5, 0)))
    m = np.arange(12, dtype=np.float32).reshape(3, 4)
    cond = np.array([True, False, True])
    assert np.array_equal(run1("Compress", {"m": m}, {"axis": 0}, {"c": cond}), m[[0, 2]])
    assert np.array_equal(run1("Compress", {"m": m}, {}, {"c": np.array([0, 1, 1], bool)}), np.array([1.0, 2.0]))
    v = np.array([1, 4, 7], np.int64)
    assert run1("BitShift", {"v": v}, {"direction": "LEFT"}, {"s": np.array([1, 2, 0], np.int64)}).tolist() == \
        [2, 16, 7]
