"""End-to-end GPU engine checks: paged chunked-prefill logits against a dense
fp32 forward, and generation through CUDA-graph decode against eager decode."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def small_cfg():
    from kapsl_sdk_b200.models.config import ModelConfig

    return ModelConfig(name="small", arch="qwen2", vocab_size=2048, hidden_size=512, intermediate_size=1024,
                       num_layers=2, num_heads=4, num_kv_heads=2, head_dim=128, rope_theta=1e6, rms_eps=1e-6,
                       qkv_bias=True, max_position=4096, bos_token_id=None, eos_token_id=None)


def make_engine(cfg, **kw):
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.models.llama import random_weights

    dev = torch.device("cuda", 0)
    w = random_weights(cfg, dev, seed=0, std=0.05)
    ecfg = EngineConfig(max_num_seqs=16, max_num_batched_tokens=kw.pop("chunk", 256), max_model_len=1024,
                        num_blocks=kw.pop("num_blocks", 512), **kw)
    return LLMEngine(cfg, weights=w, device=dev, engine_cfg=ecfg)


def test_chunked_prefill_logits_match_dense():
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.llama import random_full_weights, reference_forward

    cfg = small_cfg()
    eng = make_engine(cfg, chunk=64)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (150, 37, 64)]
    for i, p in enumerate(prompts):
        eng.add_request(f"r{i}", p, SamplingParams.greedy(4))
    # run prefill chunk by chunk; collect logits when each prompt completes
    got = {}
    while len(got) < len(prompts):
        batch = eng.scheduler.schedule()
        if batch.admitted:
            eng.runner.admit(batch.admitted)
        done = [s for s, n in batch.prefill if s.num_computed + n >= s.length]
        lg = eng.runner.logits(batch)
        for s in batch.decode:
            s.num_computed += 1
        for s, n in batch.prefill:
            s.num_computed += n
        nd = len(batch.decode)
        for r, s in enumerate(batch.decode):
            s.output_ids.append(int(lg[r].argmax()))
        for r, s in enumerate(done):  # rows after the decode rows: prompt-completing chunks
            got[s.request_id] = lg[nd + r].cpu()
            s.output_ids.append(int(lg[nd + r].argmax()))
    full = list(random_full_weights(cfg, torch.device("cuda", 0), seed=0, std=0.05))
    emb = full[0][1].cpu()
    head = full[1][1].cpu()
    layers = [{k: v.cpu() for k, v in t.items()} for kind, t in full[2:]]
    for i, p in enumerate(prompts):
        exp = reference_forward(cfg, layers, emb, head, torch.ones(cfg.hidden_size), p)[-1]
        a = got[f"r{i}"]
        err = (a - exp).abs().max().item()
        assert err < 0.05 * exp.abs().max().item() + 0.02, (i, err)


def test_generate_graph_matches_eager():
    from kapsl_sdk_b200.llm.sequence import SamplingParams

    cfg = small_cfg()
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (40, 100, 17, 250, 3)]
    outs = []
    for graphs in (True, False):
        eng = make_engine(cfg, use_cuda_graph=graphs)
        outs.append(eng.generate(prompts, SamplingParams.greedy(24, ignore_eos=True)))
        assert all(len(o) == 24 for o in outs[-1])
        if graphs:
            assert eng.runner.stats["graph_steps"] > 0
        eng.shutdown()
    # eager decode uses the graphs' batch bucket and split-KV count, and every
    # kernel is row-independent, so padding must not change a single token
    assert outs[0] == outs[1]


def test_overlapped_steps_match_serial_steps():
    """Launching step k+1 before step k's tokens reach the host (decode inputs
    taken from the previous step's sampler output on the device) gives the same
    tokens as one step at a time: same batches (all requests admitted at once,
    equal lengths), seeded top-k/top-p sampling with repetition penalty."""
    from kapsl_sdk_b200.llm.sequence import SamplingParams

    cfg = small_cfg()
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (40, 300, 17, 129, 3, 64)]
    outs = []
    for overlap in (False, True):
        eng = make_engine(cfg, overlap_steps=overlap)
        seqs = [eng.add_request(f"r{i}", p, SamplingParams(max_new_tokens=20, temperature=0.8, top_k=40, top_p=0.9,
                                                             repetition_penalty=1.1, seed=11 + i, ignore_eos=True))
                for i, p in enumerate(prompts)]
        while eng.has_unfinished():
            eng.step()
        assert all(len(s.output_ids) == 20 and s.pending is None for s in seqs)
        outs.append([s.output_ids for s in seqs])
        eng.shutdown()
    assert outs[0] == outs[1]


def test_prefix_cache_reuse_and_preemption():
    from kapsl_sdk_b200.llm.sequence import SamplingParams

    cfg = small_cfg()
    eng = make_engine(cfg, use_cuda_graph=False)
    base = list(range(100, 196))  # 96 tokens = 6 full blocks
    a = eng.generate([base + [1, 2, 3]], SamplingParams.greedy(8))[0]
    seq = eng.add_request("again", base + [1, 2, 3], SamplingParams.greedy(8))
    while eng.has_unfinished():
        eng.step()
    assert seq.num_cached_prefix == 96
    assert seq.output_ids == a


@pytest.mark.parametrize("mode", ["recompute", "swap"])
def test_preemption_keeps_sampler_state_and_kv(mode):
    """Too few KV blocks force preemptions.  (1) The LCG state of each preempted
    sequence, read back from its device slot, equals its seed advanced once per
    sampled token, so it continues the same random stream when it resumes.
    (2) Greedy outputs mostly match a roomy pool (the decode split-KV count
    follows the batch size, so a near-tie can flip a token and the rest of
    that sequence; page contents are checked bit for bit in the pool test)."""
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.ops import reference as ref

    cfg = small_cfg()
    prompts = [list(range(50 + i, 150 + i)) for i in range(6)]
    eng = make_engine(cfg, num_blocks=24, preemption=mode)
    seen = []
    orig = eng._apply_preemptions

    def spy(batch):
        orig(batch)
        seen.extend((s, s.rng_state, len(s.output_ids)) for s in batch.preempted)

    eng._apply_preemptions = spy
    p = SamplingParams(max_new_tokens=40, temperature=0.8, top_k=40, top_p=0.9, ignore_eos=True)
    seqs = [eng.add_request(f"r{i}", q, p) for i, q in enumerate(prompts)]
    while eng.has_unfinished():
        eng.step()
    assert all(len(s.output_ids) == 40 for s in seqs)
    assert any(n > 0 for _, _, n in seen), "no sequence was preempted after sampling"
    for s, st, n in seen:
        x = ref.seed_state(None, s.request_id, s.seq_id)
        for _ in range(n):
            x = (x * 6364136223846793005 + 1) & ((1 << 64) - 1)
        assert st == x, (s.request_id, n)
    st = eng.kv_stats()
    if mode == "swap":
        assert st["swap_out_total"] > 0 and st["swap_in_total"] == st["swap_out_total"] and not eng._swapped_kv

    g = SamplingParams.greedy(40, ignore_eos=True)
    want = make_engine(cfg).generate(prompts, g)
    tight = make_engine(cfg, num_blocks=24, preemption=mode)
    got = tight.generate(prompts, g)
    assert tight.kv_stats()["preemptions"] > 0
    agree = sum(int(a == b) for x, y in zip(got, want) for a, b in zip(x, y))
    assert agree >= 0.75 * sum(len(w) for w in want), (agree, got, want)
    assert sum(int(x == y) for x, y in zip(got, want)) >= 4, (got, want)


def test_kv_pool_offload_restore_bitwise():
    """Swap-out gathers pages into pinned host memory and swap-in scatters them
    into other pages, both with the block-copy kernel: bit-exact round trip."""
    from kapsl_sdk_b200.llm.kv_cache import KVLayout, KVPool

    pool = KVPool(KVLayout(num_layers=3, num_kv_heads=2, head_dim=128, block_size=16), 40, "cuda:0")
    pool.storage.copy_(torch.randn(pool.storage.shape, device="cuda:0").to(torch.bfloat16))
    before = pool.storage.clone()
    host = pool.offload([5, 9, 2, 31])
    torch.cuda.synchronize()
    assert host.is_pinned()
    assert torch.equal(host.to("cuda:0"), before[:, :, [5, 9, 2, 31]])
    pool.restore(host, [11, 3, 7, 0])
    torch.cuda.synchronize()
    assert torch.equal(pool.storage[:, :, [11, 3, 7, 0]], before[:, :, [5, 9, 2, 31]])
    untouched = [b for b in range(40) if b not in (11, 3, 7, 0)]
    assert torch.equal(pool.storage[:, :, untouched], before[:, :, untouched])


def test_rollback_regenerates_greedy():
    """Rollback keeps the KV below the cut and resets the slot's penalty counts;
    greedy decoding regenerates the tokens that were cut."""
    from kapsl_sdk_b200.llm.sequence import SamplingParams

    cfg = small_cfg()
    prompt = list(range(100, 300))
    g = SamplingParams(max_new_tokens=16, temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=1.3,
                       ignore_eos=True)
    full = make_engine(cfg).generate([prompt], g)[0]
    eng = make_engine(cfg)
    seq = eng.add_request("r", prompt, g)
    while len(seq.output_ids) < 10:
        eng.step()
    assert eng.rollback("r", len(prompt) + 4) == 1
    assert seq.output_ids == full[:4]
    while eng.has_unfinished():
        eng.step()
    assert seq.output_ids == full
