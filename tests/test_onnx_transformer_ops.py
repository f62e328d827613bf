"""Transformer-graph ONNX operators in the interpreter (standard Attention and
RotaryEmbedding, and the com.microsoft fused ops of optimized exports) against
NumPy statements of their definitions."""
import os
import tempfile

import numpy as np
import pytest

from kapsl_sdk_b200.loaders.onnx import Node, OnnxGraph, encode_model, read_model

rng = np.random.default_rng(5)


def run1(op, feeds: dict, attrs=None, inits=None, n_out=1, names=None):
    ins = names or (list(feeds) + list(inits or {}))
    outs = [f"y{i}" for i in range(n_out)]
    blob = encode_model([Node(op, ins, outs, attrs=attrs or {})], list(feeds), outs, inits or {})
    p = os.path.join(tempfile.mkdtemp(), "m.onnx")
    open(p, "wb").write(blob)
    res = OnnxGraph(read_model(p)).run(feeds)
    return [res[o].numpy() for o in outs] if n_out > 1 else res[outs[0]].numpy()


def softmax(v):
    e = np.exp(v - v.max(-1, keepdims=True))
    return e / e.sum(-1, keepdims=True)


def np_attention(q, k, v, scale, bias=None):  # [B, H, L, D] with matching heads
    s = q @ np.swapaxes(k, -1, -2) * scale
    if bias is not None:
        s = s + bias
    return softmax(s) @ v, s


@pytest.mark.parametrize("three_d", [False, True])
def test_attention_gqa_causal_past_and_mask(three_d):
    B, hq, hk, L, P, D = 2, 4, 2, 3, 2, 8
    q = rng.standard_normal((B, hq, L, D)).astype(np.float32)
    k = rng.standard_normal((B, hk, L, D)).astype(np.float32)
    v = rng.standard_normal((B, hk, L, D)).astype(np.float32)
    pk = rng.standard_normal((B, hk, P, D)).astype(np.float32)
    pv = rng.standard_normal((B, hk, P, D)).astype(np.float32)
    mask = rng.random((1, 1, L, P + L)) > 0.2
    mask[..., 0] = True
    kk = np.repeat(np.concatenate([pk, k], 2), hq // hk, 1)
    vv = np.repeat(np.concatenate([pv, v], 2), hq // hk, 1)
    bias = np.where(mask, 0.0, -np.inf) + np.where(np.tril(np.ones((L, P + L))) > 0, 0.0, -np.inf)
    want, _ = np_attention(q, kk, vv, 0.3, bias)
    attrs = {"is_causal": 1, "scale": 0.3, "qk_matmul_output_mode": 0}
    feeds = {"q": q, "k": k, "v": v, "m": mask, "pk": pk, "pv": pv}
    if three_d:
        feeds.update(q=q.transpose(0, 2, 1, 3).reshape(B, L, hq * D), k=k.transpose(0, 2, 1, 3).reshape(B, L, hk * D),
                     v=v.transpose(0, 2, 1, 3).reshape(B, L, hk * D))
        attrs.update(q_num_heads=hq, kv_num_heads=hk)
        want = want.transpose(0, 2, 1, 3).reshape(B, L, hq * D)
    y, pres_k, pres_v, qk = run1("Attention", feeds, attrs, n_out=4)
    assert np.allclose(y, want, atol=1e-5)
    assert np.allclose(pres_k, np.concatenate([pk, k], 2)) and np.allclose(pres_v, np.concatenate([pv, v], 2))
    assert np.allclose(qk, q @ np.swapaxes(kk, -1, -2) * 0.3, atol=1e-5)  # mode 0: the scaled scores


def test_attention_softcap_and_additive_mask():
    q = rng.standard_normal((1, 2, 4, 8)).astype(np.float32)
    k = rng.standard_normal((1, 2, 5, 8)).astype(np.float32)
    v = rng.standard_normal((1, 2, 5, 8)).astype(np.float32)
    m = rng.standard_normal((4, 5)).astype(np.float32)
    s = q @ np.swapaxes(k, -1, -2) / np.sqrt(8) + m
    s = 2.0 * np.tanh(s / 2.0)
    y = run1("Attention", {"q": q, "k": k, "v": v, "m": m}, {"softcap": 2.0})
    assert np.allclose(y, softmax(s) @ v, atol=1e-5)


@pytest.mark.parametrize("interleaved", [0, 1])
def test_rotary_embedding(interleaved):
    B, H, S, D, rot = 2, 3, 4, 8, 6
    x = rng.standard_normal((B, H, S, D)).astype(np.float32)
    pos = np.array([[0, 1, 2, 3], [5, 6, 7, 8]], np.int64)
    ang = np.arange(10)[:, None] * (1.0 / 10000 ** (np.arange(rot // 2) / (rot // 2)))[None]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    c, s_ = cos[pos][:, None], sin[pos][:, None]
    xr = x[..., :rot]
    if interleaved:
        x1, x2 = xr[..., 0::2], xr[..., 1::2]
        out = np.stack([x1 * c - x2 * s_, x2 * c + x1 * s_], -1).reshape(xr.shape)
    else:
        x1, x2 = xr[..., :rot // 2], xr[..., rot // 2:]
        out = np.concatenate([x1 * c - x2 * s_, x2 * c + x1 * s_], -1)
    want = np.concatenate([out, x[..., rot:]], -1)
    got = run1("RotaryEmbedding", {"x": x, "c": cos, "s": sin, "p": pos},
               {"interleaved": interleaved, "rotary_embedding_dim": rot})
    assert np.allclose(got, want, atol=1e-5)
    x3 = x.transpose(0, 2, 1, 3).reshape(B, S, H * D)  # the 3-D form with num_heads
    got3 = run1("RotaryEmbedding", {"x": x3, "c": cos, "s": sin, "p": pos},
                {"interleaved": interleaved, "rotary_embedding_dim": rot, "num_heads": H})
    assert np.allclose(got3, want.transpose(0, 2, 1, 3).reshape(B, S, H * D), atol=1e-5)


def test_skip_and_simplified_layer_norms():
    x = rng.standard_normal((2, 3, 16)).astype(np.float32)
    skip = rng.standard_normal((2, 3, 16)).astype(np.float32)
    g, b, bias = (rng.standard_normal(16).astype(np.float32) for _ in range(3))
    s = x + skip + bias
    ln = (s - s.mean(-1, keepdims=True)) / np.sqrt(s.var(-1, keepdims=True) + 1e-6) * g + b
    y, _, _, ssum = run1("SkipLayerNormalization", {"x": x, "s": skip}, {"epsilon": 1e-6},
                         {"g": g, "b": b, "bias": bias}, n_out=4)
    assert np.allclose(y, ln, atol=1e-4) and np.allclose(ssum, s, atol=1e-6)
    rms = s / np.sqrt((s * s).mean(-1, keepdims=True) + 1e-6) * g
    y, _, _, _ = run1("SkipSimplifiedLayerNormalization", {"x": x, "s": skip}, {"epsilon": 1e-6},
                      {"g": g, "bias": bias}, n_out=4)
    assert np.allclose(y, rms, atol=1e-4)
    y, _ = run1("SimplifiedLayerNormalization", {"x": x}, {"epsilon": 1e-6}, {"g": g}, n_out=2)
    assert np.allclose(y, x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * g, atol=1e-4)


def test_gelu_family_and_bias_add():
    from scipy.special import erf
    x = rng.standard_normal((3, 8)).astype(np.float32)
    b = rng.standard_normal(8).astype(np.float32)
    v = x + b
    tanh_gelu = 0.5 * v * (1 + np.tanh(np.sqrt(2 / np.pi) * (v + 0.044715 * v ** 3)))
    assert np.allclose(run1("FastGelu", {"x": x}, {}, {"b": b}), tanh_gelu, atol=1e-5)
    assert np.allclose(run1("BiasGelu", {"x": x}, {}, {"b": b}), 0.5 * v * (1 + erf(v / np.sqrt(2))), atol=1e-5)
    assert np.allclose(run1("QuickGelu", {"x": x}, {"alpha": 1.5}), x / (1 + np.exp(-1.5 * x)), atol=1e-6)
    skip = rng.standard_normal((3, 8)).astype(np.float32)
    assert np.allclose(run1("BiasAdd", {"x": x}, {}, {"b": b, "s": skip}), x + b + skip)


def test_multi_head_attention_with_padding_bias_and_past():
    B, S, P, H, D = 2, 3, 2, 2, 4
    q = rng.standard_normal((B, S, H * D)).astype(np.float32)
    k = rng.standard_normal((B, S, H * D)).astype(np.float32)
    v = rng.standard_normal((B, S, H * D)).astype(np.float32)
    bias = rng.standard_normal(3 * H * D).astype(np.float32) * 0.1
    pk = rng.standard_normal((B, H, P, D)).astype(np.float32)
    pv = rng.standard_normal((B, H, P, D)).astype(np.float32)
    lens = np.array([5, 3], np.int32)

    def heads(t):
        return t.reshape(B, S, H, D).transpose(0, 2, 1, 3)

    qh, kh, vh = heads(q + bias[:8]), heads(k + bias[8:16]), heads(v + bias[16:])
    kk, vv = np.concatenate([pk, kh], 2), np.concatenate([pv, vh], 2)
    s = qh @ np.swapaxes(kk, -1, -2) / np.sqrt(D)
    keep = (np.arange(P + S)[None, :] < lens[:, None])[:, None, None, :] & \
        (np.arange(P + S)[None, :] <= np.arange(S)[:, None] + P)
    s = np.where(keep, s, -10000.0)
    want = (softmax(s) @ vv).transpose(0, 2, 1, 3).reshape(B, S, H * D)
    feeds = {"q": q, "k": k, "v": v, "bias": bias, "kpm": lens}
    y, pres_k, _ = run1("MultiHeadAttention", dict(feeds, pk=pk, pv=pv), {"num_heads": H, "unidirectional": 1},
                        n_out=3, names=["q", "k", "v", "bias", "kpm", "", "pk", "pv"])
    assert np.allclose(y, want, atol=1e-5) and np.allclose(pres_k, kk, atol=1e-6)


@pytest.mark.parametrize("bits,with_zp", [(4, False), (4, True), (8, True), (2, False)])
def test_matmul_nbits(bits, with_zp):
    K, N, bs = 96, 5, 32
    nb = K // bs
    q = rng.integers(0, 1 << bits, (N, nb, bs))
    per = 8 // bits
    packed = np.zeros((N, nb, bs // per), np.uint8)
    for j in range(per):
        packed |= (q[:, :, j::per] << (bits * j)).astype(np.uint8)
    scales = (rng.random((N, nb)) * 0.1 + 0.01).astype(np.float32)
    zp = rng.integers(0, 1 << bits, (N, nb)) if with_zp else np.full((N, nb), 1 << (bits - 1))
    W = ((q - zp[:, :, None]) * scales[:, :, None]).reshape(N, K)
    A = rng.standard_normal((3, K)).astype(np.float32)
    inits = {"B": packed.reshape(N, nb, -1), "s": scales.reshape(-1)}
    names = ["A", "B", "s"]
    if with_zp:
        zbytes = (nb * bits + 7) // 8
        zpk = np.zeros((N, zbytes), np.uint8)
        for bidx in range(nb):
            zpk[:, (bidx * bits) // 8] |= (zp[:, bidx] << ((bidx * bits) % 8)).astype(np.uint8)
        inits["z"] = zpk.reshape(-1)
        names.append("z")
    got = run1("MatMulNBits", {"A": A}, {"K": K, "N": N, "bits": bits, "block_size": bs}, inits, names=names)
    assert np.allclose(got, A @ W.T, atol=1e-4)


def np_rotary(x, cos, sin, pos):  # x [B, H, S, D] non-interleaved over the full head
    c, s_ = cos[pos][:, None], sin[pos][:, None]
    h = x.shape[-1] // 2
    return np.concatenate([x[..., :h] * c - x[..., h:] * s_, x[..., h:] * c + x[..., :h] * s_], -1)


def test_contrib_rotary_embedding_with_start_position():
    B, S, H, D = 2, 3, 2, 8
    x = rng.standard_normal((B, S, H * D)).astype(np.float32)
    ang = np.arange(16)[:, None] * (1.0 / 10000 ** (np.arange(D // 2) / (D // 2)))[None]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    blob = encode_model([Node("RotaryEmbedding", ["x", "p", "c", "s"], ["y"], attrs={"num_heads": H},
                              domain="com.microsoft")], ["x", "p", "c", "s"], ["y"], {})
    p = os.path.join(tempfile.mkdtemp(), "m.onnx")
    open(p, "wb").write(blob)
    m = read_model(p)
    assert m.nodes[0].domain == "com.microsoft"
    got = OnnxGraph(m).run({"x": x, "p": np.array([4], np.int64), "c": cos, "s": sin})["y"].numpy()
    pos = np.tile(np.arange(4, 4 + S), (B, 1))
    xh = x.reshape(B, S, H, D).transpose(0, 2, 1, 3)
    want = np_rotary(xh, cos, sin, pos).transpose(0, 2, 1, 3).reshape(B, S, H * D)
    assert np.allclose(got, want, atol=1e-5)


@pytest.mark.parametrize("S,window", [(1, -1), (3, -1), (1, 3)])
def test_group_query_attention(S, window):
    B, hq, hk, D, Pmax = 2, 4, 2, 8, 6
    past_len = np.array([4, 2]) if S == 1 else np.array([0, 0])
    seqlens = (past_len + S - 1).astype(np.int32)
    total = int((past_len + S).max())
    q = rng.standard_normal((B, S, hq * D)).astype(np.float32)
    k = rng.standard_normal((B, S, hk * D)).astype(np.float32)
    v = rng.standard_normal((B, S, hk * D)).astype(np.float32)
    pk = rng.standard_normal((B, hk, Pmax, D)).astype(np.float32)
    pv = rng.standard_normal((B, hk, Pmax, D)).astype(np.float32)
    ang = np.arange(16)[:, None] * (1.0 / 10000 ** (np.arange(D // 2) / (D // 2)))[None]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    feeds = {"q": q, "k": k, "v": v, "pk": pk, "pv": pv, "sl": seqlens, "tot": np.array(total, np.int32),
             "c": cos, "s": sin}
    attrs = {"num_heads": hq, "kv_num_heads": hk, "do_rotary": 1, "local_window_size": window}
    blob = encode_model([Node("GroupQueryAttention", list(feeds), ["y", "pk_o", "pv_o"], attrs=attrs,
                              domain="com.microsoft")], list(feeds), ["y", "pk_o", "pv_o"], {})
    p = os.path.join(tempfile.mkdtemp(), "m.onnx")
    open(p, "wb").write(blob)
    res = OnnxGraph(read_model(p)).run(feeds)
    y = res["y"].numpy()
    for b in range(B):
        P = past_len[b]
        pos = (P + np.arange(S))[None]
        qh = np_rotary(q[b:b + 1].reshape(1, S, hq, D).transpose(0, 2, 1, 3), cos, sin, pos)[0]
        kh = np_rotary(k[b:b + 1].reshape(1, S, hk, D).transpose(0, 2, 1, 3), cos, sin, pos)[0]
        vh = v[b].reshape(S, hk, D).transpose(1, 0, 2)
        kk = np.concatenate([pk[b, :, :P], kh], 1)
        vv = np.concatenate([pv[b, :, :P], vh], 1)
        assert np.allclose(res["pk_o"].numpy()[b, :, :P + S], kk, atol=1e-5)
        kk, vv = np.repeat(kk, hq // hk, 0), np.repeat(vv, hq // hk, 0)
        sc = qh @ np.swapaxes(kk, -1, -2) / np.sqrt(D)
        qpos, kpos = P + np.arange(S), np.arange(P + S)
        keep = kpos[None, :] <= qpos[:, None]
        if window > 0:
            keep &= kpos[None, :] > qpos[:, None] - window
        sc = np.where(keep[None], sc, -np.inf)
        want = (softmax(sc) @ vv).transpose(1, 0, 2).reshape(S, hq * D)
        assert np.allclose(y[b], want, atol=1e-5)
