"""Tensor-parallel sharding on the CPU: the per-rank slices (padded query heads,
padded FFN width) add up to the unsharded layer."""
import torch

from kapsl_sdk_b200.models.config import ModelConfig
from kapsl_sdk_b200.models.llama import ShardPlan, ffn_shard_size, random_layer, shard_layer


def _mlp(x, gu, down):
    F = gu.shape[0] // 2
    g = gu.view(F // 128, 2, 128, -1)  # interleaved [gate 128 | up 128] blocks
    gate, up = g[:, 0].reshape(F, -1), g[:, 1].reshape(F, -1)
    a = x @ gate.T
    return (a * torch.sigmoid(a) * (x @ up.T)) @ down.T


def test_ffn_padding_sums_to_full():
    cfg = ModelConfig(hidden_size=256, intermediate_size=1152, num_heads=4, num_kv_heads=2, head_dim=64)
    gen = torch.Generator().manual_seed(0)
    full = {k: v.float() for k, v in random_layer(cfg, 0, gen, "cpu", std=0.05).items()}
    x = torch.randn(5, 256)
    g, u = x @ full["gate"].T, x @ full["up"].T
    ref = (g * torch.sigmoid(g) * u) @ full["down"].T
    for tp in (2, 4, 8):
        fl = ffn_shard_size(cfg, tp)
        assert fl % 128 == 0 and fl * tp >= 1152
        tot = torch.zeros_like(ref)
        for r in range(tp):
            lw = shard_layer(cfg, ShardPlan.make(cfg, tp, r), full, "cpu", dtype=torch.float32)
            assert lw.w_gu.shape == (2 * fl, 256) and lw.w_down.shape == (256, fl)
            tot += _mlp(x, lw.w_gu, lw.w_down)
        torch.testing.assert_close(tot, ref, atol=1e-4, rtol=1e-4)


def test_qwen_ffn_over_eight_ranks():
    from kapsl_sdk_b200.models.config import get_preset

    cfg = get_preset("qwen2.5-7b")
    assert ffn_shard_size(cfg, 8) == 2432 and ffn_shard_size(cfg, 4) == 4736 and ffn_shard_size(cfg, 1) == 18944


def test_padded_query_heads_cover_every_head_once():
    cfg = ModelConfig(num_heads=28, num_kv_heads=4, head_dim=128, hidden_size=3584)
    seen = []
    for r in range(8):
        p = ShardPlan.make(cfg, 8, r)
        assert p.heads_local == 4
        seen += [h for h in p.local_q_heads() if h >= 0]
    assert sorted(seen) == list(range(28))
