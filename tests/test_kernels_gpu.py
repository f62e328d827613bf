"""Numerics of every sm_100a kernel against plain fp32 PyTorch restatements."""
import math
import random

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    from kapsl_sdk_b200._ext import cuda_ops

    cuda_ops()  # must load: no silent fallback on a GPU box
    return torch.device("cuda", 0)


def close(a, b, atol, rtol=0.02):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs()
    tol = atol + rtol * b.abs()
    assert bool((err <= tol).all()), f"max err {err.max().item():.4g} (worst rel {(err / (b.abs() + 1e-6)).max():.3g})"


def test_rmsnorm(dev):
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.ops import reference as ref

    for H in (512, 3584, 8192):
        x = torch.randn(37, H, device=dev, dtype=torch.bfloat16)
        w = torch.randn(H, device=dev, dtype=torch.bfloat16)
        out = ops.rmsnorm(x, w, 1e-6)
        exp, _ = ref.rmsnorm(x.cpu(), w.cpu(), 1e-6)
        close(out, exp, 0.03)
        r = torch.randn_like(x)
        r0 = r.clone()
        out = ops.rmsnorm(x, w, 1e-6, residual=r)
        exp, s = ref.rmsnorm(x.cpu(), w.cpu(), 1e-6, residual=r0.cpu())
        close(out, exp, 0.05)
        close(r, s, 0.03)


def test_rope_kv_write(dev):
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.ops import reference as ref

    Hq, Hkv, D, T = 7, 2, 128, 45
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=dev, dtype=torch.bfloat16)
    orig = qkv.clone()
    pos = torch.randint(0, 4000, (T,), device=dev, dtype=torch.int32)
    cs = ref.rope_cos_sin(4096, D, 1e6, device=dev)
    nblocks = 20
    kc = torch.zeros(nblocks, Hkv, 16, D, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(nblocks * 16, device=dev)[:T].long()
    slots[3] = -1
    ops.rope_kv_write(qkv, pos, slots, cs, kc, vc, Hq, Hkv, D)
    q_exp = ref.apply_rope(orig[:, :Hq * D].view(T, Hq, D).cpu(), pos.cpu(), cs.cpu())
    k_exp = ref.apply_rope(orig[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D).cpu(), pos.cpu(), cs.cpu())
    close(qkv[:, :Hq * D].view(T, Hq, D), q_exp, 0.03)
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        b, o = divmod(s, 16)
        close(kc[b, :, o], k_exp[t], 0.03)
        close(vc[b, :, o], orig[t, (Hq + Hkv) * D:].view(Hkv, D), 0.0)


def test_silu_mul_and_embedding(dev):
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.ops import reference as ref

    x = torch.randn(19, 2 * 1408, device=dev, dtype=torch.bfloat16)
    close(ops.silu_mul(x), ref.silu_mul(x.cpu()), 0.03)
    table = torch.randn(1000, 512, device=dev, dtype=torch.bfloat16)
    ids = torch.tensor([0, 5, 999, 1500, 250], device=dev, dtype=torch.int32)
    out = ops.embedding(ids, table, vocab_start=250)
    exp = torch.zeros(5, 512, dtype=torch.bfloat16)
    for i, t in enumerate(ids.tolist()):
        if 250 <= t < 1250:
            exp[i] = table[t - 250].cpu()
    close(out, exp, 0.0)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 4608, 3584), (2048, 3584, 512), (7, 1536, 1024),
                                   (64, 152064 // 8, 256), (1, 896, 4736)])
def test_gemm_plain(dev, M, N, K):
    from kapsl_sdk_b200 import ops

    a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K)
    out = ops.linear(a, b)
    exp = a.float() @ b.float().T
    close(out, exp, 0.02, 0.02)
    out32 = ops.linear(a, b, out_dtype=torch.float32)
    close(out32, exp, 0.005, 0.005)


def test_gemm_epilogues(dev):
    from kapsl_sdk_b200 import ops

    M, N, K = 333, 1024, 768
    a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K)
    bias = torch.randn(N, device=dev, dtype=torch.bfloat16)
    exp = a.float() @ b.float().T
    close(ops.linear(a, b, bias=bias), exp + bias.float(), 0.03)
    r = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
    r0 = r.float().clone()
    ops.linear(a, b, residual=r, out=r)  # in place
    close(r, exp + r0, 0.05)
    # SwiGLU over interleaved gate/up
    F = 512
    g = torch.randn(F, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K)
    u = torch.randn(F, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K)
    wgu = ops.interleave_gate_up(g, u)
    out = ops.linear(a, wgu, swiglu=True)
    gg, uu = a.float() @ g.float().T, a.float() @ u.float().T
    close(out, gg * torch.sigmoid(gg) * uu, 0.03)


@pytest.mark.parametrize("splits,bn", [(2, 256), (4, 128), (3, 256)])
def test_gemm_splitk(dev, splits, bn):
    from kapsl_sdk_b200 import ops

    M, N, K = 64, 512, 2048
    a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K)
    exp = a.float() @ b.float().T
    close(ops.linear(a, b, force_bn=bn, force_splits=splits), exp, 0.02)
    r = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
    r0 = r.float().clone()
    ops.linear(a, b, residual=r, out=r, force_bn=bn, force_splits=splits)
    close(r, exp + r0, 0.05)
    F = 256
    g = torch.randn(F, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K)
    u = torch.randn(F, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K)
    out = ops.linear(a, ops.interleave_gate_up(g, u), swiglu=True, force_splits=splits)
    gg, uu = a.float() @ g.float().T, a.float() @ u.float().T
    close(out, gg * torch.sigmoid(gg) * uu, 0.03)


def _paged_setup(dev, lens, Hkv, nblocks_extra=7, seed=0):
    torch.manual_seed(seed)
    rnd = random.Random(seed)
    D = 128
    need = sum((L + 15) // 16 for L in lens)
    nb = need + nblocks_extra
    kc = torch.randn(nb, Hkv, 16, D, device=dev, dtype=torch.bfloat16)
    vc = torch.randn(nb, Hkv, 16, D, device=dev, dtype=torch.bfloat16)
    perm = list(range(nb))
    rnd.shuffle(perm)
    maxb = max((L + 15) // 16 for L in lens) + 2
    bt = torch.zeros(len(lens), maxb, dtype=torch.int32)
    tables = []
    p = 0
    for i, L in enumerate(lens):
        n = (L + 15) // 16
        tbl = perm[p:p + n]
        p += n
        bt[i, :n] = torch.tensor(tbl)
        tables.append(tbl)
    return kc, vc, bt.to(dev), tables


@pytest.mark.parametrize("Hq,Hkv", [(28, 4), (32, 8), (8, 1), (64, 8), (16, 1)])
@pytest.mark.parametrize("splits", [1, 3])
def test_decode_attention(dev, Hq, Hkv, splits):
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.ops import reference as ref

    lens = [1, 17, 300, 1025, 64, 5]
    kc, vc, bt, tables = _paged_setup(dev, lens, Hkv)
    B, D = len(lens), 128
    q = torch.randn(B, Hq * D, device=dev, dtype=torch.bfloat16)
    ctx = torch.tensor(lens, dtype=torch.int32, device=dev)
    out = ops.decode_attention(q, kc, vc, bt, ctx, Hq, Hkv, num_splits=splits)
    scale = 1 / math.sqrt(D)
    for i, L in enumerate(lens):
        k = ref.gather_paged(kc.cpu(), tables[i], L)
        v = ref.gather_paged(vc.cpu(), tables[i], L)
        exp = ref.attention(q[i].view(1, Hq, D).cpu(), k, v, scale, L - 1)
        close(out[i].view(Hq, D), exp[0], 0.02)


@pytest.mark.parametrize("Hq,Hkv", [(28, 4), (8, 8)])
def test_prefill_attention(dev, Hq, Hkv):
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.ops import reference as ref

    # (existing context, chunk length) per sequence
    specs = [(0, 130), (200, 64), (1000, 77), (16, 1), (0, 300)]
    lens = [c + n for c, n in specs]
    kc, vc, bt, tables = _paged_setup(dev, lens, Hkv, seed=1)
    D = 128
    T = sum(n for _, n in specs)
    q = torch.randn(T, Hq * D, device=dev, dtype=torch.bfloat16)
    out = torch.zeros(T, Hq * D, device=dev, dtype=torch.bfloat16)
    seq_info, work = [], []
    t = 0
    for s, (c, n) in enumerate(specs):
        seq_info.append((t, n, c + n, s))
        t += n
    work = ops.prefill_work([n for _, n in specs])
    ops.prefill_attention(q, kc, vc, torch.tensor(work, dtype=torch.int32, device=dev),
                          torch.tensor(seq_info, dtype=torch.int32, device=dev), bt, Hq, Hkv, out)
    scale = 1 / math.sqrt(D)
    for s, (c, n) in enumerate(specs):
        k = ref.gather_paged(kc.cpu(), tables[s], c + n)
        v = ref.gather_paged(vc.cpu(), tables[s], c + n)
        q0 = seq_info[s][0]
        exp = ref.attention(q[q0:q0 + n].view(n, Hq, D).cpu(), k, v, scale, c)
        close(out[q0:q0 + n].view(n, Hq, D), exp, 0.02)


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (28, 4), (8, 8)])
def test_prefill_attention_tc(dev, Hq, Hkv):
    """The tcgen05 prefill kernel against the fp32 statement (same cases as the mma.sync kernel)."""
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.ops import reference as ref

    specs = [(0, 130), (200, 64), (1000, 77), (16, 1), (0, 300)]
    lens = [c + n for c, n in specs]
    kc, vc, bt, tables = _paged_setup(dev, lens, Hkv, seed=1)
    D = 128
    T = sum(n for _, n in specs)
    q = torch.randn(T, Hq * D, device=dev, dtype=torch.bfloat16)
    out = torch.zeros(T, Hq * D, device=dev, dtype=torch.bfloat16)
    seq_info = []
    t = 0
    for s, (c, n) in enumerate(specs):
        seq_info.append((t, n, c + n, s))
        t += n
    work = ops.prefill_work([n for _, n in specs], tile=ops.prefill_tc_tile(Hq, Hkv))
    ops.prefill_attention_tc(q, kc, vc, torch.tensor(work, dtype=torch.int32, device=dev),
                             torch.tensor(seq_info, dtype=torch.int32, device=dev), bt, Hq, Hkv, out)
    torch.cuda.synchronize()
    assert ops.check_errors(torch.device(dev)) == 0
    scale = 1 / math.sqrt(D)
    for s, (c, n) in enumerate(specs):
        k = ref.gather_paged(kc.cpu(), tables[s], c + n)
        v = ref.gather_paged(vc.cpu(), tables[s], c + n)
        q0 = seq_info[s][0]
        exp = ref.attention(q[q0:q0 + n].view(n, Hq, D).cpu(), k, v, scale, c)
        close(out[q0:q0 + n].view(n, Hq, D), exp, 0.02)


def test_sampler_matches_reference(dev):
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.ops import reference as ref

    V, B = 152064, 6
    torch.manual_seed(3)
    logits = torch.randn(B, V) * 3
    params = [(0.0, 0, 1.0), (0.7, 40, 0.9), (1.0, 5, 1.0), (0.5, 1, 0.5), (1.3, 200, 0.95), (0.8, 0, 0.8)]
    states = [ref.seed_state(None, f"req-{i}", i + 1) for i in range(B)]
    temp = torch.tensor([p[0] for p in params], dtype=torch.float32, device=dev)
    topk = torch.tensor([p[1] for p in params], dtype=torch.int32, device=dev)
    topp = torch.tensor([p[2] for p in params], dtype=torch.float32, device=dev)
    rng = torch.tensor([s - (1 << 64) if s >= 1 << 63 else s for s in states], dtype=torch.int64, device=dev)
    out = torch.zeros(B, dtype=torch.int32, device=dev)
    # row 5 has top_k 0: the whole vocabulary in the reference's order (T=0.8, top_p 0.8 over 152k
    # random logits keeps a nucleus of ~100k ids)
    ops.sample(logits.to(dev).clone(), temp, topk, topp, rng, out, full_scratch=ops.sample_full_scratch(V, dev, 4),
               full_ctas=4)
    for i in range(B):
        tok, st = ref.sample_next_token(logits[i].numpy(), *params[i], states[i])
        assert int(out[i]) == tok, (i, int(out[i]), tok)
        assert int(rng[i]) & ((1 << 64) - 1) == st, i  # the LCG advanced exactly as the reference's


def test_sampler_one_pass_rows_match_reference(dev):
    """Many rows through the one-pass top-k gather (k <= 256 over a large
    vocabulary, including rows whose tail is not a multiple of four): every
    draw and LCG step equals the reference sampler's."""
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.ops import reference as ref

    g = torch.Generator().manual_seed(11)
    for V in (152064, 19013):
        B = 24
        logits = torch.randn(B, V, generator=g) * 2.5
        logits[3, 100:200] = 9.0  # ties at the top: the lower id sorts first
        ks = torch.randint(1, 257, (B,), generator=g).tolist()
        ts = (torch.rand(B, generator=g) * 1.2 + 0.3).tolist()
        ps = (torch.rand(B, generator=g) * 0.5 + 0.5).tolist()
        ts[0] = 0.0  # a greedy row
        states = [ref.seed_state(None, f"r{V}-{i}", i + 7) for i in range(B)]
        temp = torch.tensor(ts, dtype=torch.float32, device=dev)
        topk = torch.tensor(ks, dtype=torch.int32, device=dev)
        topp = torch.tensor(ps, dtype=torch.float32, device=dev)
        rng = torch.tensor([s - (1 << 64) if s >= 1 << 63 else s for s in states], dtype=torch.int64, device=dev)
        out = torch.zeros(B, dtype=torch.int32, device=dev)
        ops.sample(logits.to(dev).clone(), temp, topk, topp, rng, out)
        for i in range(B):
            tok, st = ref.sample_next_token(logits[i].numpy(), ts[i], ks[i], ps[i], states[i])
            assert int(out[i]) == tok, (V, i, int(out[i]), tok)
            assert int(rng[i]) & ((1 << 64) - 1) == st, (V, i)


def test_sampler_sparse_penalty_matches_dense(dev):
    """The occurrence lists (ids that occurred, per slot) give the same penalised
    draws as scanning the dense counts, over many rows and parameter mixes."""
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.ops import reference as ref

    V, B = 32000, 64
    g = torch.Generator().manual_seed(9)
    logits = torch.randn(B, V, generator=g) * 2
    hist = [torch.randint(0, V, (int(n),), generator=g).tolist() for n in torch.randint(0, 300, (B,), generator=g)]
    for i in range(B):  # make some penalised ids the top candidates
        for t in hist[i][:3]:
            logits[i, t] = 8.0
    counts = torch.zeros(B, V, dtype=torch.int32, device=dev)
    occ = torch.zeros(B, 512, dtype=torch.int32, device=dev)
    occ_n = torch.zeros(B, dtype=torch.int32, device=dev)
    rows = torch.tensor([i for i in range(B) for _ in hist[i]], dtype=torch.int32, device=dev)
    ids = torch.tensor([t for i in range(B) for t in hist[i]], dtype=torch.int32, device=dev)
    ops.count_tokens(counts, rows, ids, occ, occ_n)
    assert occ_n.tolist() == [len(set(h)) for h in hist]
    temp = torch.tensor([[0.0, 0.7, 1.2][i % 3] for i in range(B)], device=dev)
    topk = torch.tensor([[1, 40, 7, 1024][i % 4] for i in range(B)], dtype=torch.int32, device=dev)
    topp = torch.tensor([[1.0, 0.9, 0.5][i % 3] for i in range(B)], device=dev)
    pen = torch.tensor([[1.15, 1.0, 2.0, 0.8][i % 4] for i in range(B)], device=dev)
    states = [ref.seed_state(None, f"p-{i}", i + 1) for i in range(B)]
    outs = []
    for sparse in (True, False):
        rng = torch.tensor([s - (1 << 64) if s >= 1 << 63 else s for s in states], dtype=torch.int64, device=dev)
        out = torch.zeros(B, dtype=torch.int32, device=dev)
        ops.sample(logits.to(dev), temp, topk, topp, rng, out, rep_penalty=pen, counts=counts,
                   occ=occ if sparse else None, occ_n=occ_n if sparse else None)
        outs.append(out.tolist())
    assert outs[0] == outs[1]
    for i in range(B):
        pl = ref.apply_repetition_penalty(logits[i].numpy(), hist[i], float(pen[i]))
        tok, _ = ref.sample_next_token(pl, float(temp[i]), int(topk[i]), float(topp[i]), states[i])
        assert outs[0][i] == tok, (i, outs[0][i], tok)


@pytest.mark.parametrize("W", [2, 8])
def test_vocab_parallel_sampler_emulated(dev, W):
    """The vocabulary-parallel path on one GPU: W 'ranks' each select over their
    slice of the logits and store their candidates into the exchange buffer
    (one buffer stands for every peer's; no flags, as after an all-gather); the
    merge kernel then draws every row.  Tokens and LCG states equal the
    reference sampler's over the whole vocabulary."""
    from kapsl_sdk_b200 import _cuda, ops
    from kapsl_sdk_b200.models.llama import vocab_slice
    from kapsl_sdk_b200.ops import reference as ref

    V, B = 152064, 33
    Vs = vocab_slice(V, W)
    g = torch.Generator().manual_seed(5)
    logits = torch.randn(B, V, generator=g) * 3
    params = [[(0.0, 0, 1.0), (0.7, 40, 0.9), (1.0, 5, 1.0), (0.5, 1, 0.5), (1.3, 1024, 0.95)][i % 5]
              for i in range(B)]
    temp = torch.tensor([p[0] for p in params], device=dev)
    topk = torch.tensor([p[1] for p in params], dtype=torch.int32, device=dev)
    topp = torch.tensor([p[2] for p in params], device=dev)
    states = [ref.seed_state(7, f"vp-{i}", i + 1) for i in range(B)]
    padded = torch.zeros(B, Vs * W)
    padded[:, :V] = logits
    cand = torch.zeros(2, W, B, 1024, 2, dtype=torch.float32, device=dev)
    err = ops.error_buffer(dev)
    err.zero_()
    rng = torch.tensor([s - (1 << 64) if s >= 1 << 63 else s for s in states], dtype=torch.int64, device=dev)
    out = torch.full((B,), -1, dtype=torch.int32, device=dev)
    ctr = torch.zeros(2, dtype=torch.int64, device=dev)
    c = _cuda
    for r in range(W):  # select on each slice; candidates land in block [0][r]
        sl = padded[:, r * Vs:(r + 1) * Vs].contiguous().to(dev)
        c.sample(sl, temp, topk, topp, None, None, None, rng, out, None, None, r * Vs, V, None, 0,
                 [cand.data_ptr()] * W, [], r, B, ctr, 0, err)
    rng2 = rng.clone()
    out2 = torch.full((B,), -1, dtype=torch.int32, device=dev)
    c.sample_merge(padded[:, :Vs].contiguous().to(dev), temp, topk, topp, None, rng2, out2, V,
                   [cand.data_ptr()] * W, W - 1, B, ctr, err)
    torch.cuda.synchronize()
    assert int(err.max()) == 0
    assert int(out.min()) == -1  # select alone draws nothing
    for i in range(B):
        tok, st = ref.sample_next_token(logits[i].numpy(), *params[i], states[i])
        assert int(out2[i]) == tok, (i, int(out2[i]), tok)
        if params[i][0] > 0:
            assert int(rng2[i]) & ((1 << 64) - 1) == st, i


def test_sampler_penalty_counts(dev):
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.ops import reference as ref

    V = 1000
    torch.manual_seed(4)
    logits = torch.randn(2, V)
    hist = [[5, 5, 9, 100, 5], [7]]
    counts = torch.zeros(3, V, dtype=torch.int32, device=dev)
    rows = torch.tensor([2] * 5 + [0], dtype=torch.int32, device=dev)
    ids = torch.tensor(hist[0] + hist[1], dtype=torch.int32, device=dev)
    ops.count_tokens(counts, rows, ids)
    slots = torch.tensor([2, 0], dtype=torch.int32, device=dev)
    states = [11, 22]
    rng = torch.zeros(3, dtype=torch.int64, device=dev)
    rng[2], rng[0] = states[0], states[1]
    out = torch.zeros(2, dtype=torch.int32, device=dev)
    temp = torch.tensor([0.0, 0.9], device=dev)
    topk = torch.tensor([0, 10], dtype=torch.int32, device=dev)
    topp = torch.tensor([1.0, 0.7], device=dev)
    pen = torch.tensor([1.3, 2.0], device=dev)
    # make penalised ids the argmax before the penalty
    logits[0, 5] = 10.0
    logits[1, 7] = 10.0
    ops.sample(logits.to(dev).clone(), temp, topk, topp, rng, out, rep_penalty=pen, counts=counts, slots=slots)
    for i in range(2):
        pl = ref.apply_repetition_penalty(logits[i].numpy(), hist[i], float(pen[i]))
        tok, st = ref.sample_next_token(pl, float(temp[i]), int(topk[i]), float(topp[i]), states[i])
        assert int(out[i]) == tok
    assert int(rng[0]) != 22  # the LCG advanced for the sampled row


@pytest.mark.parametrize("bn", [256, 224, 192, 128])
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (300, 4608, 3584), (2048, 3584, 512), (520, 1000, 192)])
def test_gemm_2sm(dev, M, N, K, bn):
    """cta_group::2 path (CTA pairs, 256 x bn tiles; N not always a multiple of bn)."""
    from kapsl_sdk_b200 import ops

    fb = 256 + bn  # force_bn > 256 selects the 2-SM kernel with tiles bn wide
    a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K)
    exp = a.float() @ b.float().T
    close(ops.linear(a, b, force_bn=fb), exp, 0.02)
    close(ops.linear(a, b, force_bn=fb, out_dtype=torch.float32), exp, 0.005, 0.005)
    bias = torch.randn(N, device=dev, dtype=torch.bfloat16)
    close(ops.linear(a, b, bias=bias, force_bn=fb), exp + bias.float(), 0.03)
    r = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
    r0 = r.float().clone()
    ops.linear(a, b, residual=r, out=r, force_bn=fb)
    close(r, exp + r0, 0.05)
    if N % 256 == 0 and bn == 256:
        F = N // 2
        g = torch.randn(F, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K)
        u = torch.randn(F, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K)
        out = ops.linear(a, ops.interleave_gate_up(g, u), swiglu=True, force_bn=512)
        gg, uu = a.float() @ g.float().T, a.float() @ u.float().T
        close(out, gg * torch.sigmoid(gg) * uu, 0.03)
