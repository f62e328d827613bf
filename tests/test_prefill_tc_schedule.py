"""The tcgen05 prefill attention kernel's schedule, restated step by step on
the CPU: head-group row packing (row r -> token r // g, head r % g), 128-key
tiles over paged KV, the masks, the two-pass softmax with the running max,
and the order in which the previous tile's P.V is folded in (o = o * c_prev +
O_prev before this tile's P is written).  The statement must equal plain
causal attention; the kernel itself is checked against it on a GPU."""
import math

import numpy as np
import pytest
import torch

from kapsl_sdk_b200.ops import prefill_tc_tile, prefill_work
from kapsl_sdk_b200.ops import reference as ref


def kernel_schedule(q, kc, vc, bt, row0, n, ctx, Hq, Hkv, scale, t0):
    """One CTA per KV head for the work item at token t0; returns {(token, head): out row}."""
    D, g = 128, Hq // Hkv
    tpc = 128 // g
    ntok = min(tpc, n - t0)
    q_last = ctx - n + t0 + ntok - 1
    ntiles = (q_last + 128) // 128
    out = {}
    log2e = 1.4426950408889634
    for kvh in range(Hkv):
        Q = np.zeros((128, D), np.float32)
        for r in range(g * tpc):
            tok, head = r // g, r % g
            if row0 + t0 + tok < q.shape[0]:
                Q[r] = q[row0 + t0 + tok, (kvh * g + head) * D:(kvh * g + head + 1) * D]
        m = np.full(128, -np.inf)
        l = np.zeros(128)
        o = np.zeros((128, D))
        corr_prev = np.zeros(128)
        O_prev = None
        for j in range(ntiles):
            pages = [bt[p] if p < (ctx + 15) // 16 else bt[0] for p in range(8 * j, 8 * j + 8)]
            K = np.concatenate([kc[b, kvh] for b in pages])  # [128 keys, D]
            V = np.concatenate([vc[b, kvh] for b in pages])
            S = Q @ K.T
            kpos = j * 128 + np.arange(128)[None, :]
            qpos = (ctx - n + t0 + np.arange(128) // g)[:, None]
            X = np.where((kpos > qpos) | (kpos >= ctx), -np.inf, S * scale * log2e)
            m_new = np.maximum(m, X.max(1))
            corr = np.exp2(m - m_new)
            if j > 0:
                o = o * corr_prev[:, None] + O_prev
            P = np.exp2(X - m_new[:, None])
            l = l * corr + P.sum(1)
            m = m_new
            corr_prev = corr
            O_prev = P.astype(np.float32) @ V
        o = o * corr_prev[:, None] + O_prev
        for r in range(g * tpc):
            tok, head = r // g, r % g
            if tok < ntok:
                out[(t0 + tok, kvh * g + head)] = o[r] / l[r]
    return out


@pytest.mark.parametrize("Hq,Hkv,ctx,n", [(8, 2, 300, 300), (7, 1, 200, 70), (12, 4, 129, 129), (4, 4, 40, 40)])
def test_schedule_equals_causal_attention(Hq, Hkv, ctx, n):
    rng = np.random.default_rng(0)
    D, nblocks = 128, 64
    kc = rng.standard_normal((nblocks, Hkv, 16, D)).astype(np.float32)
    vc = rng.standard_normal((nblocks, Hkv, 16, D)).astype(np.float32)
    bt = rng.permutation(nblocks)[:(ctx + 15) // 16 + 8].tolist()
    q = rng.standard_normal((n + 5, Hq * D)).astype(np.float32) * 0.3
    row0, scale = 5, 1 / math.sqrt(D)
    tile = prefill_tc_tile(Hq, Hkv)
    got = {}
    for s, t0 in prefill_work([n], tile):
        got.update(kernel_schedule(q, kc, vc, bt, row0, n, ctx, Hq, Hkv, scale, t0))
    assert len(got) == n * Hq
    K = np.concatenate([kc[b].transpose(1, 0, 2) for b in bt])[:ctx]  # [ctx, Hkv, D]
    V = np.concatenate([vc[b].transpose(1, 0, 2) for b in bt])[:ctx]
    want = ref.attention(torch.from_numpy(q[row0:row0 + n].reshape(n, Hq, D)), torch.from_numpy(K.copy()),
                         torch.from_numpy(V.copy()), scale, ctx - n).numpy()
    for (t, h), v in got.items():
        assert np.allclose(v, want[t, h], atol=1e-4), (t, h)
