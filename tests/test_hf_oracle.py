"""Each supported HF model family, built tiny with random weights by
transformers and saved with save_pretrained, loaded by this runtime's
checkpoint loader and served by the CPU engine: prompt logits and greedy
tokens must match transformers' own forward (the oracle)."""
import pytest
import torch

transformers = pytest.importorskip("transformers")

GEOM = dict(vocab_size=320, hidden_size=64, intermediate_size=128, num_hidden_layers=3, num_attention_heads=4,
            num_key_value_heads=2, head_dim=16, max_position_embeddings=512, pad_token_id=0, bos_token_id=1,
            eos_token_id=2)

FAMILIES = {
    "llama": ("LlamaConfig", "LlamaForCausalLM", {}),
    "mistral": ("MistralConfig", "MistralForCausalLM", {"sliding_window": None}),
    "qwen2": ("Qwen2Config", "Qwen2ForCausalLM", {}),
    "qwen3": ("Qwen3Config", "Qwen3ForCausalLM", {}),
    "phi3": ("Phi3Config", "Phi3ForCausalLM", {}),
    "gemma": ("GemmaConfig", "GemmaForCausalLM", {}),
    "gemma2": ("Gemma2Config", "Gemma2ForCausalLM", {"sliding_window": 6, "attn_logit_softcapping": 8.0,
                                                     "final_logit_softcapping": 5.0, "query_pre_attn_scalar": 24}),
    "mixtral": ("MixtralConfig", "MixtralForCausalLM", {"num_local_experts": 4, "num_experts_per_tok": 2}),
    "llama3-rope": ("LlamaConfig", "LlamaForCausalLM", {"rope_theta": 500000.0, "rope_scaling": {
        "rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
        "original_max_position_embeddings": 64}}),
}


def build(family, tmp_path):
    cname, mname, extra = FAMILIES[family]
    cfg = getattr(transformers, cname)(**{**GEOM, **extra})
    torch.manual_seed(0)
    model = getattr(transformers, mname)(cfg).float().eval()
    with torch.no_grad():
        for name, p in model.named_parameters():
            base = 1.0 if "norm" in name and not family.startswith("gemma") else 0.0
            p.copy_(torch.randn_like(p) * (0.3 if "norm" in name else 0.08) + base)
    path = tmp_path / family
    model.save_pretrained(str(path), safe_serialization=True)
    # eager attention: transformers' SDPA path leaves out Gemma 2's attention soft-capping
    oracle = getattr(transformers, mname).from_pretrained(str(path), attn_implementation="eager").float().eval()
    return oracle, str(path)


@pytest.mark.parametrize("family", sorted(FAMILIES))
def test_family_matches_transformers(family, tmp_path):
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.loaders.hf import load_hf_model

    hf, path = build(family, tmp_path)
    cfg, model, _ = load_hf_model(path, "cpu")
    prompt = [5 + (7 * i) % 300 for i in range(23)]
    with torch.no_grad():
        want_logits = hf(torch.tensor([prompt])).logits[0, -1].float()
        toks = list(prompt)
        for _ in range(8):
            toks.append(int(hf(torch.tensor([toks])).logits[0, -1].argmax()))
    eng = LLMEngine(cfg, weights=model, device="cpu", engine_cfg=EngineConfig(
        max_num_seqs=2, max_num_batched_tokens=16, max_model_len=128, num_blocks=32), seed=0)
    from kapsl_sdk_b200.llm.scheduler import ScheduledBatch
    from kapsl_sdk_b200.llm.sequence import Sequence

    got = eng.generate([prompt], SamplingParams.greedy(8, ignore_eos=True))[0]
    assert got == toks[len(prompt):], (family, got, toks[len(prompt):])
    # prompt logits through the paged runner (chunked prefill over 16-token chunks)
    seq = Sequence(seq_id=99, request_id="x", prompt_ids=prompt, params=SamplingParams.greedy(1))
    seq.block_ids = eng.allocator.allocate(2)
    logits = None
    for c0 in range(0, len(prompt), 16):
        n = min(16, len(prompt) - c0)
        seq.num_computed = c0
        b = ScheduledBatch(prefill=[(seq, n)])
        logits = eng.runner.logits(b)
    assert torch.allclose(logits[-1].float(), want_logits, atol=2e-4, rtol=1e-4), \
        (family, (logits[-1] - want_logits).abs().max())


def test_gemma2_gguf_round_trip_matches_transformers(tmp_path):
    """HF Gemma 2 -> this runtime's tensor stream -> GGUF (norms with the +1
    folded in, soft-caps and window in metadata) -> served tokens equal
    transformers' greedy continuation."""
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.loaders.gguf import load_gguf_model, write_gguf_model
    from kapsl_sdk_b200.loaders.hf import iter_hf_full
    from kapsl_sdk_b200.models.config import ModelConfig

    hf, path = build("gemma2", tmp_path)
    cfg = ModelConfig.from_hf_config(path + "/config.json")
    g = str(tmp_path / "g2.gguf")
    write_gguf_model(g, cfg, iter_hf_full(path, cfg), quant="f32", arch="gemma2")
    c2, m2, _ = load_gguf_model(g, "cpu")
    assert (c2.attn_softcap, c2.final_softcap, c2.sliding_window, c2.act) == (8.0, 5.0, 6, "gelu_tanh")
    prompt = [5 + (7 * i) % 300 for i in range(23)]
    with torch.no_grad():
        toks = list(prompt)
        for _ in range(8):
            toks.append(int(hf(torch.tensor([toks])).logits[0, -1].argmax()))
    eng = LLMEngine(c2, weights=m2, device="cpu", engine_cfg=EngineConfig(
        max_num_seqs=2, max_num_batched_tokens=16, max_model_len=128, num_blocks=32), seed=0)
    assert eng.generate([prompt], SamplingParams.greedy(8, ignore_eos=True))[0] == toks[len(prompt):]


@pytest.mark.parametrize("family", ["llama", "qwen2", "mixtral", "llama3-rope"])
def test_gpu_oracle_matches_transformers(family, tmp_path):
    """models.llama.reference_forward is the fp32 oracle of the GPU kernel
    tests; on the GPU families it must equal transformers' forward."""
    from kapsl_sdk_b200.loaders.hf import iter_hf_full
    from kapsl_sdk_b200.models.config import ModelConfig
    from kapsl_sdk_b200.models.llama import reference_forward

    hf, path = build(family, tmp_path)
    cfg = ModelConfig.from_hf_config(path + "/config.json")
    items = list(iter_hf_full(path, cfg))
    d = dict((k, v) for k, v in items if k != "layer")
    layers = [v for k, v in items if k == "layer"]
    prompt = [5 + (7 * i) % 300 for i in range(23)]
    got = reference_forward(cfg, layers, d["embed"], d["lm_head"], d["final_norm"], prompt)
    with torch.no_grad():
        want = hf(torch.tensor([prompt])).logits[0].float()
    assert torch.allclose(got, want, atol=2e-4, rtol=1e-4), (got - want).abs().max()
