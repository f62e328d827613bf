"""GGUF Q4_K on the GPU: the quantizer matches the Python reference byte for
byte, the dequantizer matches the Python reference, and the fused
dequant-in-mainloop GEMM matches x @ dequant(W).T (fp32), including split-K,
the residual epilogue, ragged token counts and a Q4_K model end to end."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _w(n, k, seed, std=0.02):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g) * std).to(torch.bfloat16)


def test_quantize_matches_reference_bytes():
    from kapsl_sdk_b200.loaders.gguf import quantize_q4_k as np_quant
    from kapsl_sdk_b200.quantization import quantize_q4_k

    w = _w(64, 1024, 0)
    w[3, :256] = 0  # an all-zero super-block
    w[5, 256:512] = torch.abs(w[5, 256:512])  # no negative values: min 0
    qw = quantize_q4_k(w.cuda(), tiled=False)
    ref = np_quant(w.float().numpy().reshape(-1)).reshape(64, -1)
    got = qw.raw.cpu().numpy()
    assert got.shape == ref.shape
    assert np.array_equal(got, ref), int((got != ref).sum())


def test_dequant_matches_reference():
    from kapsl_sdk_b200.loaders.gguf import dequant_q4_k
    from kapsl_sdk_b200.quantization import quantize_q4_k

    w = _w(32, 2048, 1)
    qw = quantize_q4_k(w.cuda(), tiled=False)
    got = qw.dequantize().float().cpu()
    ref = torch.from_numpy(dequant_q4_k(qw.raw.cpu().numpy().reshape(-1))).view(32, 2048)
    w2 = _w(256, 512, 2)
    qr, qt = quantize_q4_k(w2.cuda(), tiled=False), quantize_q4_k(w2.cuda())  # row-major / tile-major
    assert qt.tiled and torch.equal(qt.row_major().cpu(), qr.raw.cpu())
    assert torch.equal(qt.dequantize(), qr.dequantize())
    torch.testing.assert_close(got, ref.to(torch.bfloat16).float(), atol=0, rtol=0)
    assert (got - w.float()).abs().max() < 0.01  # a 4-bit code of N(0, 0.02) values


@pytest.mark.parametrize("M,N,K", [(1, 128, 256), (5, 384, 1024), (64, 1280, 8192), (100, 256, 4096),
                                   (128, 1000, 768), (300, 512, 2048), (1030, 256, 512)])
@pytest.mark.parametrize("tiled", [True, False])
def test_gemm_q4k(M, N, K, tiled):
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.quantization import quantize_q4_k

    dev = torch.device("cuda", 0)
    qw = quantize_q4_k(_w(N, K, M + N).to(dev), tiled=tiled)
    x = (torch.randn(M, K, generator=torch.Generator().manual_seed(K)) * 0.5).to(dev, torch.bfloat16)
    y = ops.linear(x, qw)
    ref = x.float() @ qw.dequantize().float().T
    err = (y.float() - ref).abs().max().item()
    assert err <= 0.02 * ref.abs().max().item() + 1e-3, err
    assert ops.check_errors(dev) == 0


def test_gemm_q4k_split_and_residual():
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200._ext import cuda_ops
    from kapsl_sdk_b200.quantization import quantize_q4_k

    dev = torch.device("cuda", 0)
    M, N, K = 48, 640, 4096
    qw = quantize_q4_k(_w(N, K, 7).to(dev))
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    res = torch.randn(M, N, device=dev).to(torch.bfloat16)
    ref = x.float() @ qw.dequantize().float().T + res.float()
    for splits in (1, 3, 16):
        out = res.clone()
        cuda_ops().gemm_q4k(x, qw.raw, out, K, out, ops._workspace(dev), splits, qw.tiled, ops.error_buffer(dev))
        err = (out.float() - ref).abs().max().item()
        assert err <= 0.02 * ref.abs().max().item() + 1e-2, (splits, err)
    assert ops.check_errors(dev) == 0


def test_q4k_model_generates():
    """A small Llama with Q4_K linear layers: greedy tokens agree with the same
    model run on the dequantized (bf16) weights."""
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.config import ModelConfig
    from kapsl_sdk_b200.models.llama import random_weights

    dev = torch.device("cuda", 0)
    cfg = ModelConfig(name="tiny-q4k", arch="llama", vocab_size=2048, hidden_size=512, intermediate_size=1536,
                      num_layers=2, num_heads=4, num_kv_heads=2, head_dim=128, rope_theta=5e5, max_position=2048,
                      weight_format="q4_k", bos_token_id=None, eos_token_id=None)
    wq = random_weights(cfg, dev, seed=0, std=0.05)
    ecfg = EngineConfig(max_num_seqs=8, max_num_batched_tokens=128, max_model_len=512, num_blocks=128)
    prompts = [list(range(5, 70)), list(range(100, 133))]
    outs_q = LLMEngine(cfg, weights=wq, device=dev, engine_cfg=ecfg).generate(
        prompts, SamplingParams.greedy(8, ignore_eos=True))
    # same weights, dequantized to bf16 tensors (gate/up re-interleaved for the bf16 path)
    from kapsl_sdk_b200 import ops

    for L in wq.layers:
        L.w_qkv, L.w_o, L.w_down = L.w_qkv.dequantize(), L.w_o.dequantize(), L.w_down.dequantize()
        gu = L.w_gu.dequantize()
        F = gu.shape[0] // 2
        L.w_gu = ops.interleave_gate_up(gu[:F], gu[F:])
    cfg.weight_format = "bf16"
    outs_b = LLMEngine(cfg, weights=wq, device=dev, engine_cfg=ecfg).generate(
        prompts, SamplingParams.greedy(8, ignore_eos=True))
    agree = sum(int(a == b) for o1, o2 in zip(outs_q, outs_b) for a, b in zip(o1, o2))
    assert agree >= 14, (outs_q, outs_b)


@pytest.mark.parametrize("tiled", [True, False])
def test_dequant_rows_matches_dequantizer(tiled):
    """The whole-matrix dequant of the large-token path gives the dequantizer's
    bf16 bits, in row order and in the interleaved gate/up (SwiGLU) order."""
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200._ext import cuda_ops
    from kapsl_sdk_b200.quantization import quantize_q4_k

    dev = torch.device("cuda", 0)
    N, K = 512, 1536
    qw = quantize_q4_k(_w(N, K, 11).to(dev), tiled=tiled)
    ref = qw.dequantize()
    got = torch.empty(N, K + 64, device=dev, dtype=torch.bfloat16)  # padded pitch
    cuda_ops().q4k_dequant_rows(qw.raw, N, K, qw.tiled, 0, got)
    assert torch.equal(got[:, :K], ref)
    inter = torch.empty(N, K, device=dev, dtype=torch.bfloat16)
    cuda_ops().q4k_dequant_rows(qw.raw, N, K, qw.tiled, N // 2, inter)
    assert torch.equal(inter, ops.interleave_gate_up(ref[:N // 2], ref[N // 2:]))


@pytest.mark.parametrize("M", [600, 1100])
def test_gemm_q4k_large_token_path(M, monkeypatch):
    """From Q4K_DEQUANT_MIN_M tokens the product runs as dequant + bf16 GEMM: plain,
    residual and SwiGLU results agree with the fp32 reference and with the fused kernel."""
    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200.quantization import quantize_q4_k

    dev = torch.device("cuda", 0)
    N, K = 1024, 2048
    qw = quantize_q4_k(_w(N, K, 5).to(dev))
    x = (torch.randn(M, K, generator=torch.Generator().manual_seed(3)) * 0.5).to(dev, torch.bfloat16)
    res = torch.randn(M, N, device=dev).to(torch.bfloat16)
    wf = qw.dequantize().float()
    ref = x.float() @ wf.T
    gate, up = ref[:, :N // 2], ref[:, N // 2:]
    ref_sw = gate * torch.sigmoid(gate) * up
    outs = {}
    monkeypatch.setattr(ops, "Q4K_DEQUANT_MIN_N", 0)
    for thr in (M, 1 << 30):  # dequant path, then the fused kernel
        monkeypatch.setattr(ops, "Q4K_DEQUANT_MIN_M", thr)
        y = ops.linear(x, qw)
        yr = ops.linear(x, qw, residual=res)
        ys = ops.linear(x, qw, swiglu=True)
        tol = 0.02 * ref.abs().max().item() + 1e-3
        assert (y.float() - ref).abs().max().item() <= tol
        assert (yr.float() - ref - res.float()).abs().max().item() <= tol + 1e-2
        assert (ys.float() - ref_sw).abs().max().item() <= 0.02 * ref_sw.abs().max().item() + 1e-3
        outs[thr] = y
    # both paths multiply the same dequantized weights; they differ only in rounding
    assert (outs[M].float() - outs[1 << 30].float()).abs().max().item() <= 0.02 * ref.abs().max().item()
    assert ops.check_errors(dev) == 0
