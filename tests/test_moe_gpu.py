"""Mixture-of-experts kernels against fp32 PyTorch oracles: router top-k,
grouped tcgen05 GEMMs over the expert-sorted rows (with and without split-K),
the combine, expert-parallel sharding (ranks emulated on one GPU), and a
Mixtral-style model through the engine against the dense fp32 forward."""
import types

import pytest
import torch

pytestmark = pytest.mark.gpu


def moe_cfg(E=8, K=2, d=512, F=1024, layers=2):
    from kapsl_sdk_b200.models.config import ModelConfig

    return ModelConfig(name="tiny-moe", arch="mixtral", vocab_size=2048, hidden_size=d, intermediate_size=F,
                       num_layers=layers, num_heads=4, num_kv_heads=2, head_dim=128, rope_theta=1e6, rms_eps=1e-5,
                       max_position=4096, num_experts=E, experts_per_token=K, bos_token_id=None, eos_token_id=None)


def _layer(cfg, dev, seed, std=0.05):
    from kapsl_sdk_b200 import ops

    g = torch.Generator().manual_seed(seed)
    E, d, F = cfg.num_experts, cfg.hidden_size, cfg.intermediate_size
    full = {"router": torch.randn(E, d, generator=g) * std * 4,
            "gate": torch.randn(E, F, d, generator=g) * std,
            "up": torch.randn(E, F, d, generator=g) * std,
            "down": torch.randn(E, d, F, generator=g) * std}
    full = {k: v.to(torch.bfloat16) for k, v in full.items()}

    def shard(e0, el):
        L = types.SimpleNamespace()
        L.w_router = full["router"].to(dev).contiguous()
        L.w_experts_gu = torch.stack([ops.interleave_gate_up(full["gate"][e], full["up"][e])
                                      for e in range(e0, e0 + el)]).to(dev).contiguous()
        L.w_experts_down = full["down"][e0:e0 + el].to(dev).contiguous()
        return L

    return full, shard


def test_moe_route():
    from kapsl_sdk_b200 import ops

    dev = torch.device("cuda", 0)
    for E, K, T in ((8, 2, 300), (60, 4, 77), (64, 8, 5)):
        x = torch.randn(T, 1024, device=dev).to(torch.bfloat16)
        wr = (torch.randn(E, 1024, device=dev) * 0.05).to(torch.bfloat16)
        ids, w = ops.moe_route(x, wr, K, renormalize=(E == 8))
        p = torch.softmax(x.float() @ wr.float().T, -1)
        tv, ti = p.topk(K, -1)
        if E == 8:
            tv = tv / tv.sum(-1, keepdim=True)
        assert torch.equal(ids.long().sort(-1).values, ti.sort(-1).values)
        torch.testing.assert_close(w.sort(-1).values, tv.sort(-1).values, atol=1e-4, rtol=1e-3)


@pytest.mark.parametrize("T", [1, 37, 300, 1030])
def test_moe_layer_matches_reference(T):
    from kapsl_sdk_b200.models.moe import MoE, reference_moe

    dev = torch.device("cuda", 0)
    cfg = moe_cfg()
    full, shard = _layer(cfg, dev, seed=T)
    moe = MoE(cfg, dev)
    moe.configure(2048)
    x = (torch.randn(T, cfg.hidden_size, device=dev)).to(torch.bfloat16)
    h0 = (torch.randn(T, cfg.hidden_size, device=dev)).to(torch.bfloat16)
    h = h0.clone()
    moe.forward(x, shard(0, cfg.num_experts), h)
    exp = reference_moe(x.cpu(), full["router"], full["gate"], full["up"], full["down"], cfg.experts_per_token)
    got = (h.float() - h0.float()).cpu()
    err = (got - exp).abs().max().item()
    assert err < 0.03 * exp.abs().max().item() + 0.02, err
    from kapsl_sdk_b200 import ops

    assert ops.check_errors(dev) == 0


def test_grouped_gemm_split_k():
    """Force split-K on the grouped GEMM and compare with the unsplit result."""
    from kapsl_sdk_b200 import ops

    dev = torch.device("cuda", 0)
    E, d, F, T, K = 4, 512, 2048, 64, 2
    g = torch.Generator().manual_seed(3)
    x = torch.randn(T, d, generator=g).to(dev, torch.bfloat16)
    wr = (torch.randn(E, d, generator=g) * 0.2).to(dev, torch.bfloat16)
    wd = (torch.randn(E * d, F, generator=g) * 0.05).to(dev, torch.bfloat16)
    ids, w = ops.moe_route(x, wr, K)
    R = ((T * K + E * 127 + 127) // 128) * 128
    seg = torch.zeros(E + 1, dtype=torch.int32, device=dev)
    pos = torch.zeros(T * K, dtype=torch.int32, device=dev)
    mt = torch.zeros(1 + R // 128, dtype=torch.int32, device=dev)
    src = torch.zeros(R, dtype=torch.int32, device=dev)
    ops.moe_permute(ids, E, 0, E, R, seg, pos, mt, src)
    hs = (torch.randn(R, F, generator=g) * 0.5).to(dev, torch.bfloat16)
    y1 = torch.zeros(R, d, dtype=torch.bfloat16, device=dev)
    y4 = torch.zeros(R, d, dtype=torch.bfloat16, device=dev)
    ops.grouped_linear(hs, wd, d, mt, y1, splits=1, bn=128)
    ops.grouped_linear(hs, wd, d, mt, y4, splits=4, bn=128)
    n = int(mt[0]) * 128
    tiles = mt[1:1 + n // 128].cpu().tolist()
    exp = torch.cat([hs[i * 128:(i + 1) * 128].float() @ wd[e * d:(e + 1) * d].float().T for i, e in enumerate(tiles)])
    torch.testing.assert_close(y1[:n].float(), exp, atol=0.05, rtol=0.02)
    torch.testing.assert_close(y4[:n].float(), exp, atol=0.05, rtol=0.02)


def test_expert_parallel_shards_sum_to_reference():
    """Two expert-parallel ranks emulated on one GPU (local-only combine):
    the ranks' partial outputs add up to the full MoE."""
    from kapsl_sdk_b200.models.moe import MoE, reference_moe

    dev = torch.device("cuda", 0)
    cfg = moe_cfg()
    full, shard = _layer(cfg, dev, seed=11)
    T = 200
    x = torch.randn(T, cfg.hidden_size, device=dev).to(torch.bfloat16)
    total = torch.zeros(T, cfg.hidden_size, device=dev)
    for r in range(2):
        fake = types.SimpleNamespace(world_size=2, rank=r, mode="nccl", all_reduce=lambda t: t, max_tokens=0)
        moe = MoE(cfg, dev, fake)
        moe.configure(512)
        h = torch.zeros(T, cfg.hidden_size, device=dev, dtype=torch.bfloat16)
        moe.forward(x, shard(r * 4, 4), h)
        total += h.float()
    exp = reference_moe(x.cpu(), full["router"], full["gate"], full["up"], full["down"], cfg.experts_per_token)
    err = (total.cpu() - exp).abs().max().item()
    assert err < 0.03 * exp.abs().max().item() + 0.02, err


def test_mixtral_engine_logits_match_dense():
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.llama import random_full_weights, random_weights, reference_forward

    cfg = moe_cfg()
    dev = torch.device("cuda", 0)
    w = random_weights(cfg, dev, seed=0, std=0.05)
    eng = LLMEngine(cfg, weights=w, device=dev,
                    engine_cfg=EngineConfig(max_num_seqs=8, max_num_batched_tokens=128, max_model_len=512,
                                            num_blocks=256))
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (90, 33)]
    outs = eng.generate(prompts, SamplingParams.greedy(6, ignore_eos=True))
    full = list(random_full_weights(cfg, dev, seed=0, std=0.05))
    emb, head = full[0][1].cpu(), full[1][1].cpu()
    layers = [{k: v.cpu() for k, v in t.items()} for kind, t in full[2:]]
    agree = 0
    for p, o in zip(prompts, outs):
        lg = reference_forward(cfg, layers, emb, head, torch.ones(cfg.hidden_size), p + o[:-1])
        ref_next = lg[len(p) - 1:].argmax(-1).tolist()
        agree += sum(int(a == b) for a, b in zip(ref_next, o))
    assert agree >= 0.8 * sum(len(o) for o in outs), agree
    eng.shutdown()
