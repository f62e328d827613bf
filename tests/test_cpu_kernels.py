"""C++ CPU kernels of the CPU backend against the fp32 PyTorch reference ops,
and the CPU model with and without them."""
import os

import numpy as np
import pytest
import torch

from kapsl_sdk_b200.ops import reference as ref


@pytest.fixture(scope="module")
def k():
    from kapsl_sdk_b200._ext import native

    return native().cpu


def test_rmsnorm_rope_silu(k):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(37, 96, generator=g)
    w = torch.randn(96, generator=g)
    out = torch.empty_like(x)
    k.rmsnorm(x.numpy(), w.numpy(), out.numpy(), 1e-5)
    torch.testing.assert_close(out, ref.rmsnorm(x, w, 1e-5)[0], atol=1e-5, rtol=1e-5)
    q = torch.randn(9, 4, 64, generator=g)
    pos = torch.randint(0, 500, (9,), generator=g)
    cs = ref.rope_cos_sin(512, 64, 10000.0)
    want = ref.apply_rope(q, pos, cs)
    k.rope(q.numpy(), pos.numpy().astype(np.int64), cs.numpy())
    torch.testing.assert_close(q, want, atol=1e-5, rtol=1e-5)
    gu = torch.randn(11, 2 * 40, generator=g)
    act = torch.empty(11, 40)
    k.silu_mul(gu.numpy(), act.numpy())
    torch.testing.assert_close(act, ref.silu_mul(gu), atol=1e-5, rtol=1e-5)


def test_paged_attention_and_kv_write(k):
    g = torch.Generator().manual_seed(1)
    Hq, Hkv, D, bs = 8, 2, 32, 16
    specs = [(0, 20), (31, 5), (7, 1)]  # (existing context, new tokens)
    nb = 40
    kc = torch.zeros(nb, Hkv, bs, D)
    vc = torch.zeros(nb, Hkv, bs, D)
    perm = torch.randperm(nb, generator=g).tolist()
    tables, row0, nq, ctx = [], [], [], []
    T = sum(n for _, n in specs)
    q = torch.randn(T, Hq, D, generator=g)
    kn, vn = torch.randn(T, Hkv, D, generator=g), torch.randn(T, Hkv, D, generator=g)
    slots = torch.empty(T, dtype=torch.int64)
    r, p = 0, 0
    for c, n in specs:
        L = c + n
        tbl = perm[p:p + (L + bs - 1) // bs]
        p += len(tbl)
        tables.append(tbl)
        for j in range(c):  # pre-existing context
            kc[tbl[j // bs], :, j % bs] = torch.randn(Hkv, D, generator=g)
            vc[tbl[j // bs], :, j % bs] = torch.randn(Hkv, D, generator=g)
        for i in range(n):
            slots[r + i] = tbl[(c + i) // bs] * bs + (c + i) % bs
        row0.append(r)
        nq.append(n)
        ctx.append(L)
        r += n
    k.kv_write(kn.numpy(), vn.numpy(), slots.numpy(), kc.numpy(), vc.numpy())
    bt = np.zeros((len(specs), max(len(t) for t in tables)), dtype=np.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    out = torch.empty(T, Hq, D)
    k.paged_attention(q.numpy(), kc.numpy(), vc.numpy(), np.array(row0, np.int64), np.array(nq, np.int64),
                      np.array(ctx, np.int64), bt, D ** -0.5, out.numpy())
    for s, (c, n) in enumerate(specs):
        kk = ref.gather_paged(kc, tables[s], c + n)
        vv = ref.gather_paged(vc, tables[s], c + n)
        want = ref.attention(q[row0[s]:row0[s] + n], kk, vv, D ** -0.5, c)
        torch.testing.assert_close(out[row0[s]:row0[s] + n], want, atol=1e-5, rtol=1e-4)


def test_cpu_model_native_matches_torch(monkeypatch):
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.config import ModelConfig

    cfg = ModelConfig(name="t", vocab_size=300, hidden_size=64, intermediate_size=128, num_layers=2, num_heads=4,
                      num_kv_heads=2, head_dim=16, max_position=512, bos_token_id=None, eos_token_id=None)
    outs = []
    for mode in ("native", "torch"):
        monkeypatch.setenv("KAPSL_CPU_KERNELS", mode)
        eng = LLMEngine(cfg, device="cpu", engine_cfg=EngineConfig(max_num_seqs=4, max_num_batched_tokens=32,
                        max_model_len=256, num_blocks=64), seed=0)
        assert (eng.model._k is not None) == (mode == "native")
        outs.append(eng.generate([list(range(3, 50)), list(range(7, 20))], SamplingParams.greedy(10, ignore_eos=True)))
    assert outs[0] == outs[1]
