"""More ONNX operators in the interpreter: Resize per the spec's coordinate modes
(golden outputs of the operator documentation's examples, and the library's
bilinear / bicubic where the two coincide), NonMaxSuppression, integer and
quantized-linear products and convolutions, normalizations, sequence utilities,
trigonometric functions and random generators, against NumPy statements."""
import os
import tempfile

import numpy as np
import pytest
import torch

from kapsl_sdk_b200.loaders.onnx import Node, OnnxGraph, encode_model, read_model

rng = np.random.default_rng(11)


def run1(op, feeds: dict, attrs=None, inits=None, n_out=1):
    ins = [k for k in list(feeds) + list(inits or {})]
    outs = [f"y{i}" for i in range(n_out)]
    blob = encode_model([Node(op, ins, outs, attrs=attrs or {})], list(feeds), outs, inits or {})
    p = os.path.join(tempfile.mkdtemp(), "m.onnx")
    open(p, "wb").write(blob)
    res = OnnxGraph(read_model(p)).run(feeds)
    return [res[o].numpy() for o in outs] if n_out > 1 else res[outs[0]].numpy()


def resize(x, attrs, scales=None, sizes=None, roi=None):
    inits = {"roi": roi if roi is not None else np.zeros(0, np.float32),
             "scales": scales if scales is not None else np.zeros(0, np.float32)}
    if sizes is not None:
        inits["sizes"] = sizes
    return run1("Resize", {"x": x}, attrs, inits)


def test_resize_golden_examples():
    x = np.array([[[[1, 2], [3, 4]]]], np.float32)
    got = resize(x, {"mode": "nearest"}, scales=np.array([1, 1, 2, 3], np.float32))
    assert np.array_equal(got[0, 0], [[1, 1, 1, 2, 2, 2], [1, 1, 1, 2, 2, 2], [3, 3, 3, 4, 4, 4], [3, 3, 3, 4, 4, 4]])
    x2 = np.array([[[[1, 2, 3, 4], [5, 6, 7, 8]]]], np.float32)
    got = resize(x2, {"mode": "linear"}, scales=np.array([1, 1, 0.6, 0.6], np.float32))
    assert np.allclose(got, [[[[2.6666665, 4.3333331]]]], atol=1e-5)
    got = resize(x2, {"mode": "nearest"}, scales=np.array([1, 1, 0.6, 0.6], np.float32))
    assert np.array_equal(got, [[[[1, 3]]]])
    got = resize(x, {"mode": "linear", "coordinate_transformation_mode": "align_corners"},
                 scales=np.array([1, 1, 2, 2], np.float32))
    want = [[1, 4 / 3, 5 / 3, 2], [5 / 3, 2, 7 / 3, 8 / 3], [7 / 3, 8 / 3, 3, 10 / 3], [3, 10 / 3, 11 / 3, 4]]
    assert np.allclose(got[0, 0], want, atol=1e-5)
    x4 = np.arange(1, 17, dtype=np.float32).reshape(1, 1, 4, 4)
    got = resize(x4, {"mode": "linear", "coordinate_transformation_mode": "tf_crop_and_resize"},
                 sizes=np.array([1, 1, 3, 3], np.int64), roi=np.array([0, 0, 0.4, 0.6, 1, 1, 0.6, 0.8], np.float32))
    assert np.allclose(got[0, 0], [[7.6, 7.9, 8.2], [8.8, 9.1, 9.4], [10.0, 10.3, 10.6]], atol=1e-5)
    got = run1("Upsample", {"x": x}, {"mode": "nearest"}, {"s": np.array([1, 1, 2, 3], np.float32)})
    assert np.array_equal(got[0, 0], [[1, 1, 1, 2, 2, 2], [1, 1, 1, 2, 2, 2], [3, 3, 3, 4, 4, 4], [3, 3, 3, 4, 4, 4]])


@pytest.mark.parametrize("mode,tmode", [("linear", "bilinear"), ("cubic", "bicubic")])
def test_resize_upsampling_matches_half_pixel_interpolation(mode, tmode):
    x = rng.standard_normal((2, 3, 5, 7)).astype(np.float32)
    got = resize(x, {"mode": mode}, sizes=np.array([2, 3, 11, 9], np.int64))
    want = torch.nn.functional.interpolate(torch.from_numpy(x), size=(11, 9), mode=tmode, align_corners=False)
    assert np.allclose(got, want.numpy(), atol=1e-5)


def test_resize_nearest_modes_and_exclude_outside():
    x = np.arange(4, dtype=np.float32).reshape(1, 1, 1, 4)
    # asymmetric with scale 1.5 maps outputs 0..5 to 0, .67, 1.33, 2, 2.67, 3.33
    for nm, want in [("floor", [0, 0, 1, 2, 2, 3]), ("ceil", [0, 1, 2, 2, 3, 3]),
                     ("round_prefer_floor", [0, 1, 1, 2, 3, 3])]:
        got = resize(x, {"mode": "nearest", "coordinate_transformation_mode": "asymmetric", "nearest_mode": nm},
                     scales=np.array([1, 1, 1, 1.5], np.float32))
        assert got[0, 0, 0].tolist() == want, nm
    got = resize(x, {"mode": "cubic", "exclude_outside": 1, "cubic_coeff_a": -0.5},
                 scales=np.array([1, 1, 1, 2], np.float32))
    assert got.shape == (1, 1, 1, 8) and abs(got[0, 0, 0, 0] - 0.0) < 0.2 and abs(got[0, 0, 0, -1] - 3.0) < 0.2


def test_non_max_suppression_golden():
    boxes = np.array([[[0, 0, 1, 1], [0, 0.1, 1, 1.1], [0, -0.1, 1, 0.9], [0, 10, 1, 11], [0, 10.1, 1, 11.1],
                       [0, 100, 1, 101]]], np.float32)
    scores = np.array([[[0.9, 0.75, 0.6, 0.95, 0.5, 0.3]]], np.float32)
    inits = {"m": np.array([3], np.int64), "iou": np.array([0.5], np.float32), "st": np.array([0.0], np.float32)}
    got = run1("NonMaxSuppression", {"b": boxes, "s": scores}, {}, inits)
    assert got.tolist() == [[0, 0, 3], [0, 0, 0], [0, 0, 5]]
    centers = np.array([[[0.5, 0.5, 1, 1], [0.5, 0.6, 1, 1], [0.5, 0.4, 1, 1], [0.5, 10.5, 1, 1],
                         [0.5, 10.6, 1, 1], [0.5, 100.5, 1, 1]]], np.float32)
    got = run1("NonMaxSuppression", {"b": centers, "s": scores}, {"center_point_box": 1}, inits)
    assert got.tolist() == [[0, 0, 3], [0, 0, 0], [0, 0, 5]]
    inits["st"] = np.array([0.7], np.float32)  # the score threshold drops 0.6 and below
    got = run1("NonMaxSuppression", {"b": boxes, "s": scores}, {}, inits)
    assert got.tolist() == [[0, 0, 3], [0, 0, 0]]


def test_integer_and_quantized_products():
    A = np.array([[11, 7, 3], [10, 6, 2], [9, 5, 1], [8, 4, 0]], np.uint8)
    B = np.array([[1, 4], [2, 5], [3, 6]], np.uint8)
    got = run1("MatMulInteger", {"a": A, "b": B}, {}, {"az": np.array(12, np.uint8), "bz": np.array(0, np.uint8)})
    assert got.dtype == np.int32 and got.tolist() == [[-38, -83], [-44, -98], [-50, -113], [-56, -128]]
    qa = rng.integers(0, 255, (3, 5)).astype(np.uint8)
    qb = rng.integers(0, 255, (5, 4)).astype(np.uint8)
    sa, za, sb, zb, sy, zy = 0.02, 113, 0.01, 114, 0.05, 118
    got = run1("QLinearMatMul", {"a": qa}, {}, {"sa": np.array(sa, np.float32), "za": np.array(za, np.uint8),
                                                "b": qb, "sb": np.array(sb, np.float32), "zb": np.array(zb, np.uint8),
                                                "sy": np.array(sy, np.float32), "zy": np.array(zy, np.uint8)})
    real = ((qa.astype(np.float64) - za) * np.float32(sa)) @ ((qb.astype(np.float64) - zb) * np.float32(sb))
    want = np.clip(np.round(real / np.float32(sy)) + zy, 0, 255).astype(np.uint8)
    assert np.array_equal(got, want)


def _conv2d_np(x, w, pads=(0, 0)):
    x = np.pad(x, ((0, 0), (0, 0), (pads[0], pads[0]), (pads[1], pads[1])))
    N, C, H, W = x.shape
    O, _, kh, kw = w.shape
    y = np.zeros((N, O, H - kh + 1, W - kw + 1))
    for i in range(y.shape[2]):
        for j in range(y.shape[3]):
            y[:, :, i, j] = np.einsum("nchw,ochw->no", x[:, :, i:i + kh, j:j + kw], w)
    return y


def test_integer_and_quantized_convolutions():
    x = rng.integers(0, 255, (1, 2, 5, 5)).astype(np.uint8)
    w = rng.integers(0, 255, (3, 2, 3, 3)).astype(np.uint8)
    xz, wz = 100, np.array([120, 128, 90], np.uint8)
    got = run1("ConvInteger", {"x": x}, {"pads": [1, 1, 1, 1]}, {"w": w, "xz": np.array(xz, np.uint8), "wz": wz})
    want = _conv2d_np(x.astype(np.float64) - xz, w.astype(np.float64) - wz.reshape(3, 1, 1, 1), (1, 1))
    assert got.dtype == np.int32 and np.array_equal(got, want.astype(np.int32))
    sx, sw, sy, zy = np.float32(0.01), np.array([0.02, 0.03, 0.01], np.float32), np.float32(0.5), 7
    bias = np.array([100, -50, 30], np.int32)
    got = run1("QLinearConv", {"x": x}, {}, {"sx": np.array(sx), "xz": np.array(xz, np.uint8), "w": w,
                                             "sw": sw, "wz": wz, "sy": np.array(sy), "zy": np.array(zy, np.uint8),
                                             "b": bias})
    acc = _conv2d_np(x.astype(np.float64) - xz, w.astype(np.float64) - wz.reshape(3, 1, 1, 1)) + \
        bias.reshape(1, 3, 1, 1)
    want = np.clip(np.round(acc * (np.float64(sx) * sw.astype(np.float64).reshape(1, 3, 1, 1)) / np.float64(sy)) + zy,
                   0, 255).astype(np.uint8)
    assert np.array_equal(got, want)


def test_normalizations():
    x = rng.standard_normal((2, 5, 3, 4)).astype(np.float32)
    for size in (3, 4):
        got = run1("LRN", {"x": x}, {"size": size, "alpha": 0.01, "beta": 0.6, "bias": 2.0})
        lo, hi = (size - 1) // 2, size - 1 - (size - 1) // 2
        sq = np.pad(x * x, ((0, 0), (lo, hi), (0, 0), (0, 0)))
        acc = sum(sq[:, i:i + 5] for i in range(size))
        assert np.allclose(got, x / (2.0 + 0.01 / size * acc) ** 0.6, atol=1e-5)
    m = x.mean(axis=(0, 2, 3), keepdims=True)
    sd = np.sqrt((x * x).mean(axis=(0, 2, 3), keepdims=True) - m * m)
    assert np.allclose(run1("MeanVarianceNormalization", {"x": x}), (x - m) / (sd + 1e-9), atol=1e-4)
    sc = rng.standard_normal(4).astype(np.float32)
    want = x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * sc
    assert np.allclose(run1("RMSNormalization", {"x": x}, {"epsilon": 1e-6}, {"s": sc}), want, atol=1e-5)
    p = 3
    got = run1("LpPool", {"x": x}, {"kernel_shape": [2, 2], "strides": [1, 2], "p": p})
    want = np.zeros((2, 5, 2, 2), np.float32)
    for i in range(2):
        for j in range(2):
            want[:, :, i, j] = (np.abs(x[:, :, i:i + 2, 2 * j:2 * j + 2]) ** p).sum((2, 3)) ** (1 / p)
    assert np.allclose(got, want, atol=1e-5)
    assert np.allclose(run1("GlobalLpPool", {"x": x}), np.sqrt((x * x).sum((2, 3), keepdims=True)), atol=1e-5)


def test_sequences_and_selection():
    x = np.arange(16, dtype=np.float32).reshape(4, 4)
    lens = np.array([4, 3, 2, 1], np.int64)
    got = run1("ReverseSequence", {"x": x}, {"time_axis": 0, "batch_axis": 1}, {"l": lens})
    want = x.copy()
    for b, L in enumerate(lens):
        want[:L, b] = x[:L, b][::-1]
    assert np.array_equal(got, want)
    u = np.array([2, 1, 1, 3, 4, 3], np.float32)
    y, idx, inv, cnt = run1("Unique", {"u": u}, {"sorted": 0}, n_out=4)
    assert y.tolist() == [2, 1, 3, 4] and idx.tolist() == [0, 1, 3, 4]
    assert inv.tolist() == [0, 1, 1, 2, 3, 2] and cnt.tolist() == [1, 2, 2, 1]
    y, idx, inv, cnt = run1("Unique", {"u": u}, {}, n_out=4)
    assert y.tolist() == [1, 2, 3, 4] and idx.tolist() == [1, 0, 3, 4]
    assert inv.tolist() == [1, 0, 0, 2, 3, 2] and cnt.tolist() == [2, 1, 2, 1]
    h = rng.standard_normal((3, 5)).astype(np.float32)
    assert np.array_equal(run1("Hardmax", {"h": h}), np.eye(5, dtype=np.float32)[h.argmax(-1)])
    assert np.array_equal(run1("EyeLike", {"e": np.zeros((3, 5), np.float32)}, {"k": 2}), np.eye(3, 5, k=2))
    m = rng.standard_normal((2, 3, 3)).astype(np.float32)
    assert np.allclose(run1("Det", {"m": m}), np.linalg.det(m), atol=1e-5)


def test_trigonometric_and_inf():
    x = np.linspace(-0.9, 0.9, 7, dtype=np.float32)
    for op, f in [("Tan", np.tan), ("Asin", np.arcsin), ("Acos", np.arccos), ("Atan", np.arctan),
                  ("Sinh", np.sinh), ("Cosh", np.cosh), ("Asinh", np.arcsinh), ("Atanh", np.arctanh)]:
        assert np.allclose(run1(op, {"x": x}), f(x), atol=1e-6), op
    assert np.allclose(run1("Acosh", {"x": x + 2}), np.arccosh(x + 2), atol=1e-6)
    v = np.array([1.0, np.inf, -np.inf, np.nan], np.float32)
    assert run1("IsInf", {"v": v}).tolist() == [False, True, True, False]
    assert run1("IsInf", {"v": v}, {"detect_negative": 0}).tolist() == [False, True, False, False]
    assert run1("CastLike", {"v": np.array([1.7, -2.2], np.float32)}, {}, {"t": np.zeros(1, np.int32)}).tolist() == \
        [1, -2]


def test_random_generators_are_seeded():
    a = run1("RandomNormal", {}, {"shape": [4000], "mean": 2.0, "scale": 0.5, "seed": 3.0})
    b = run1("RandomNormal", {}, {"shape": [4000], "mean": 2.0, "scale": 0.5, "seed": 3.0})
    assert a.dtype == np.float32 and np.array_equal(a, b) and abs(a.mean() - 2.0) < 0.05 and abs(a.std() - 0.5) < 0.05
    u = run1("RandomUniformLike", {"t": np.zeros((50, 40), np.float32)}, {"low": -1.0, "high": 3.0, "seed": 1.0})
    assert u.shape == (50, 40) and u.min() >= -1 and u.max() <= 3 and abs(u.mean() - 1.0) < 0.1
    p = np.full(5000, 0.25, np.float32)
    bern = run1("Bernoulli", {"p": p}, {"seed": 2.0})
    assert set(np.unique(bern).tolist()) <= {0.0, 1.0} and abs(bern.mean() - 0.25) < 0.03


def test_grid_sample_identity_grid():
    x = rng.standard_normal((1, 2, 4, 5)).astype(np.float32)
    ys, xs = np.meshgrid(np.linspace(-1, 1, 4), np.linspace(-1, 1, 5), indexing="ij")
    grid = np.stack([xs, ys], -1)[None].astype(np.float32)
    got = run1("GridSample", {"x": x, "g": grid}, {"align_corners": 1})
    assert np.allclose(got, x, atol=1e-5)
