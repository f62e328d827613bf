"""ONNX control flow (If, Loop, Scan with subgraphs that read outer-scope names)
and recurrent layers (RNN, GRU, LSTM) in the interpreter, against NumPy
statements of the ONNX operator spec; graphs go through the protobuf encoder
and decoder."""
import os
import tempfile

import numpy as np
import pytest

from kapsl_sdk_b200.loaders.onnx import Node, OnnxGraph, OnnxModel, encode_model, read_model

rng = np.random.default_rng(7)


def run(nodes, feeds: dict, outs: list, inits=None):
    blob = encode_model(nodes, list(feeds), outs, inits or {})
    p = os.path.join(tempfile.mkdtemp(), "m.onnx")
    open(p, "wb").write(blob)
    res = OnnxGraph(read_model(p)).run(feeds)
    return [res[o].numpy() for o in outs]


def test_if_picks_branch_and_reads_outer_scope():
    x = rng.standard_normal((3, 4)).astype(np.float32)
    then_g = OnnxModel([Node("Add", ["x", "x"], ["t"])], [], ["t"], {})
    else_g = OnnxModel([Node("Mul", ["x", "k"], ["e"])], [], ["e"], {"k": np.array(3.0, np.float32)})
    node = Node("If", ["c"], ["y"], attrs={"then_branch": then_g, "else_branch": else_g})
    (y,) = run([node], {"c": np.array(True), "x": x}, ["y"])
    assert np.allclose(y, 2 * x)
    (y,) = run([node], {"c": np.array([False]), "x": x}, ["y"])
    assert np.allclose(y, 3 * x)


def test_loop_with_trip_count_condition_and_scan_outputs():
    # body: acc_out = acc + x * i; cond_out = acc_out.sum() < limit; scan out: acc_out
    body = OnnxModel([Node("Cast", ["i"], ["fi"], attrs={"to": 1}),
                      Node("Mul", ["x", "fi"], ["xi"]),
                      Node("Add", ["acc", "xi"], ["acc_out"]),
                      Node("ReduceSum", ["acc_out"], ["s"], attrs={"keepdims": 0}),
                      Node("Less", ["s", "limit"], ["cond_out"]),
                      Node("Identity", ["acc_out"], ["scan"])],
                     ["i", "cond_in", "acc"], ["cond_out", "acc_out", "scan"], {})
    x = np.array([1.0, 2.0], np.float32)
    node = Node("Loop", ["M", "", "acc0"], ["acc_final", "scans"], attrs={"body": body})
    acc_final, scans = run([node], {"M": np.array(5, np.int64), "acc0": np.zeros(2, np.float32), "x": x,
                                    "limit": np.array(1e9, np.float32)}, ["acc_final", "scans"])
    want = [x * sum(range(i + 1)) for i in range(5)]
    assert np.allclose(acc_final, want[-1]) and np.allclose(scans, np.stack(want))
    # the condition ends the loop early: sums 0, 3, 9, 18 -> stops once >= 9
    node = Node("Loop", ["M", "c0", "acc0"], ["acc_final", "scans"], attrs={"body": body})
    acc_final, scans = run([node], {"M": np.array(100, np.int64), "c0": np.array(True),
                                    "acc0": np.zeros(2, np.float32), "x": x, "limit": np.array(9.0, np.float32)},
                           ["acc_final", "scans"])
    assert scans.shape == (3, 2) and np.allclose(acc_final, x * 3)


@pytest.mark.parametrize("direction", [0, 1])
def test_scan_running_sum_with_directions_and_axes(direction):
    body = OnnxModel([Node("Add", ["s_in", "xt"], ["s_out"]), Node("Identity", ["s_out"], ["y"])],
                     ["s_in", "xt"], ["s_out", "y"], {})
    x = rng.standard_normal((4, 3)).astype(np.float32)  # scanned along axis 1 (3 steps of shape [4])
    node = Node("Scan", ["s0", "x"], ["s_final", "ys"],
                attrs={"body": body, "num_scan_inputs": 1, "scan_input_axes": [1],
                       "scan_input_directions": [direction], "scan_output_axes": [-1]})
    s_final, ys = run([node], {"s0": np.zeros(4, np.float32), "x": x}, ["s_final", "ys"])
    cols = x[:, ::-1] if direction else x
    want = np.cumsum(cols, axis=1)
    assert np.allclose(ys, want, atol=1e-6) and np.allclose(s_final, x.sum(1), atol=1e-6)


# ------------------------------------------------------------- recurrent layers
def sig(v):
    return 1 / (1 + np.exp(-v))


def np_recurrent(op, X, W, R, B, lens, h0, c0=None, P=None, direction="forward", lbr=0, clip=None):
    """The ONNX RNN / GRU / LSTM equations, one batch row and time step at a time."""
    seq, batch, _ = X.shape
    nd = 2 if direction == "bidirectional" else 1
    H = R.shape[-1]
    G = {"RNN": 1, "GRU": 3, "LSTM": 4}[op]
    Y = np.zeros((seq, nd, batch, H), np.float32)
    Yh = np.zeros((nd, batch, H), np.float32)
    Yc = np.zeros((nd, batch, H), np.float32)
    cl = (lambda v: np.clip(v, -clip, clip)) if clip else (lambda v: v)
    for d in range(nd):
        rev = direction == "reverse" or d == 1
        Wb, Rb = (B[d][:G * H], B[d][G * H:]) if B is not None else (np.zeros(G * H), np.zeros(G * H))
        for b in range(batch):
            h = h0[d, b].copy() if h0 is not None else np.zeros(H, np.float32)
            c = c0[d, b].copy() if c0 is not None else np.zeros(H, np.float32)
            L = lens[b]
            for s in range(L):
                t = L - 1 - s if rev else s
                xt = X[t, b]
                if op == "RNN":
                    h = np.tanh(cl(W[d] @ xt + Wb + R[d] @ h + Rb))
                elif op == "GRU":
                    z = sig(cl(W[d][:H] @ xt + Wb[:H] + R[d][:H] @ h + Rb[:H]))
                    r = sig(cl(W[d][H:2 * H] @ xt + Wb[H:2 * H] + R[d][H:2 * H] @ h + Rb[H:2 * H]))
                    if lbr:
                        hh = np.tanh(cl(W[d][2 * H:] @ xt + Wb[2 * H:] + r * (R[d][2 * H:] @ h + Rb[2 * H:])))
                    else:
                        hh = np.tanh(cl(W[d][2 * H:] @ xt + Wb[2 * H:] + R[d][2 * H:] @ (r * h) + Rb[2 * H:]))
                    h = (1 - z) * hh + z * h
                else:
                    g = W[d] @ xt + Wb + R[d] @ h + Rb
                    pi, po, pf = (P[d][:H], P[d][H:2 * H], P[d][2 * H:]) if P is not None else (0, 0, 0)
                    i = sig(cl(g[:H] + pi * c))
                    f = sig(cl(g[2 * H:3 * H] + pf * c))
                    c = f * c + i * np.tanh(cl(g[3 * H:]))
                    o = sig(cl(g[H:2 * H] + po * c))
                    h = o * np.tanh(c)
                Y[t, d, b] = h
            Yh[d, b] = h
            Yc[d, b] = c
    return Y, Yh, Yc


@pytest.mark.parametrize("op", ["RNN", "GRU", "LSTM"])
@pytest.mark.parametrize("direction", ["forward", "reverse", "bidirectional"])
def test_recurrent_layers_match_the_spec(op, direction):
    seq, batch, inp, H = 5, 3, 4, 6
    G = {"RNN": 1, "GRU": 3, "LSTM": 4}[op]
    nd = 2 if direction == "bidirectional" else 1
    X = rng.standard_normal((seq, batch, inp)).astype(np.float32)
    W = (rng.standard_normal((nd, G * H, inp)) * 0.4).astype(np.float32)
    R = (rng.standard_normal((nd, G * H, H)) * 0.4).astype(np.float32)
    B = (rng.standard_normal((nd, 2 * G * H)) * 0.2).astype(np.float32)
    lens = np.array([5, 2, 4], np.int32)
    h0 = (rng.standard_normal((nd, batch, H)) * 0.3).astype(np.float32)
    feeds = {"X": X, "W": W, "R": R, "B": B, "L": lens, "h0": h0}
    ins = ["X", "W", "R", "B", "L", "h0"]
    extra = {}
    if op == "LSTM":
        extra = {"c0": (rng.standard_normal((nd, batch, H)) * 0.3).astype(np.float32),
                 "P": (rng.standard_normal((nd, 3 * H)) * 0.2).astype(np.float32)}
        feeds.update(extra)
        ins += ["c0", "P"]
    attrs = {"hidden_size": H, "direction": direction}
    if op == "GRU":
        attrs["linear_before_reset"] = 1
    outs = ["Y", "Yh", "Yc"] if op == "LSTM" else ["Y", "Yh"]
    got = run([Node(op, ins, outs, attrs=attrs)], feeds, outs)
    want = np_recurrent(op, X, W, R, B, lens, h0, extra.get("c0"), extra.get("P"), direction,
                        lbr=attrs.get("linear_before_reset", 0))
    for g, w in zip(got, want):
        assert np.allclose(g, w, atol=1e-5), np.abs(g - w).max()


def test_gru_default_reset_and_lstm_layout1_without_optional_inputs():
    seq, batch, inp, H = 4, 2, 3, 5
    X = rng.standard_normal((seq, batch, inp)).astype(np.float32)
    W = (rng.standard_normal((1, 3 * H, inp)) * 0.5).astype(np.float32)
    R = (rng.standard_normal((1, 3 * H, H)) * 0.5).astype(np.float32)
    got = run([Node("GRU", ["X", "W", "R"], ["Y", "Yh"], attrs={"hidden_size": H, "clip": 0.5})],
              {"X": X, "W": W, "R": R}, ["Y", "Yh"])
    want = np_recurrent("GRU", X, W, R, None, [seq] * batch, None, clip=0.5)
    assert np.allclose(got[0], want[0], atol=1e-5) and np.allclose(got[1], want[1], atol=1e-5)
    W4 = (rng.standard_normal((1, 4 * H, inp)) * 0.5).astype(np.float32)
    R4 = (rng.standard_normal((1, 4 * H, H)) * 0.5).astype(np.float32)
    Xb = np.ascontiguousarray(X.transpose(1, 0, 2))  # layout 1: [batch, seq, input]
    got = run([Node("LSTM", ["X", "W", "R"], ["Y", "Yh", "Yc"], attrs={"hidden_size": H, "layout": 1})],
              {"X": Xb, "W": W4, "R": R4}, ["Y", "Yh", "Yc"])
    Y, Yh, Yc = np_recurrent("LSTM", X, W4, R4, None, [seq] * batch, None)
    assert np.allclose(got[0], Y.transpose(2, 0, 1, 3), atol=1e-5)
    assert np.allclose(got[1], Yh.transpose(1, 0, 2), atol=1e-5)
    assert np.allclose(got[2], Yc.transpose(1, 0, 2), atol=1e-5)


def test_subgraph_ops_are_checked_at_load():
    bad = OnnxModel([Node("NoSuchOp", ["x"], ["y"])], [], ["y"], {})
    node = Node("If", ["c"], ["y"], attrs={"then_branch": bad, "else_branch": bad})
    blob = encode_model([node], ["c", "x"], ["y"], {})
    p = os.path.join(tempfile.mkdtemp(), "m.onnx")
    open(p, "wb").write(blob)
    with pytest.raises(ValueError, match="NoSuchOp"):
        OnnxGraph(read_model(p))
