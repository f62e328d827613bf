"""Kernel micro-benchmarks / profiling drivers for the sm_100a kernels.

    python -m kapsl_sdk_b200.utils.kernel_bench gemm M N K [--epi plain|bias|residual|swiglu] [--time]
    python -m kapsl_sdk_b200.utils.kernel_bench gemm_q4k M N K [--time]
    python -m kapsl_sdk_b200.utils.kernel_bench moe T E D F [--time]
    python -m kapsl_sdk_b200.utils.kernel_bench decode B CTX HQ HKV [--time]
    python -m kapsl_sdk_b200.utils.kernel_bench prefill S CHUNK HQ HKV [--time]
    python -m kapsl_sdk_b200.utils.kernel_bench sample B V [--time]

Without ``--time`` each command launches the kernel 3 times (a capture target
for ncu: ``-k regex:<kernel> -s 2 -c 1``).  With ``--time`` it reports the
CUDA-event time over 20 launches after 3 warm-ups and the achieved
FLOP/s or bytes/s.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import random

import torch


def _time(fn, iters: int = 20) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_gemm(M, N, K, epi, timed, cublas=False, iters=20):
    from .. import ops

    dev = torch.device("cuda", 0)
    a = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K)
    kw = {}
    if epi == "bias":
        kw["bias"] = torch.randn(N, device=dev, dtype=torch.bfloat16)
    elif epi == "residual":
        kw["residual"] = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
        kw["out"] = kw["residual"]
    elif epi == "swiglu":
        kw["swiglu"] = True
    fn = lambda: ops.linear(a, b, **kw)
    if not timed:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return {"kernel": "gemm", "M": M, "N": N, "K": K}
    ms = _time(fn, iters)
    r = {"kernel": "gemm", "M": M, "N": N, "K": K, "epi": epi, "iters": iters, "ms": ms,
         "tflops": 2 * M * N * K / ms / 1e9}
    if cublas:  # the library GEMM of the same plain product, timed the same way
        ms_lib = _time(lambda: torch.nn.functional.linear(a, b), iters)
        r.update(cublas_ms=ms_lib, cublas_tflops=2 * M * N * K / ms_lib / 1e9, ratio=ms_lib / ms)
    return r


def bench_decode(B, ctx, hq, hkv, timed):
    from .. import ops

    dev = torch.device("cuda", 0)
    nb_seq = (ctx + 15) // 16
    nblocks = B * nb_seq
    kc = torch.randn(nblocks, hkv, 16, 128, device=dev, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    perm = list(range(nblocks))
    random.Random(0).shuffle(perm)  # randomly permuted block tables
    bt = torch.tensor(perm, dtype=torch.int32, device=dev).view(B, nb_seq)
    q = torch.randn(B, hq * 128, device=dev, dtype=torch.bfloat16)
    lens = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    fn = lambda: ops.decode_attention(q, kc, vc, bt, lens, hq, hkv, out=out, max_ctx=ctx)
    if not timed:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return {"kernel": "decode_attention", "B": B, "ctx": ctx}
    ms = _time(fn)
    nbytes = 2 * B * ctx * hkv * 128 * 2
    return {"kernel": "decode_attention", "B": B, "ctx": ctx, "hq": hq, "hkv": hkv, "ms": ms,
            "GBps": nbytes / ms / 1e6}


def bench_prefill(S, chunk, hq, hkv, timed):
    from .. import ops

    dev = torch.device("cuda", 0)
    nb_seq = (chunk + 15) // 16
    kc = torch.randn(S * nb_seq, hkv, 16, 128, device=dev, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = torch.arange(S * nb_seq, dtype=torch.int32, device=dev).view(S, nb_seq)
    q = torch.randn(S * chunk, hq * 128, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    info = torch.tensor([(s * chunk, chunk, chunk, s) for s in range(S)], dtype=torch.int32, device=dev)
    tc = os.environ.get("KAPSL_PREFILL_TC") == "1"  # the tcgen05 kernel instead of the mma.sync one
    tile = ops.prefill_tc_tile(hq, hkv) if tc else 64
    work = torch.tensor(ops.prefill_work([chunk] * S, tile=tile), dtype=torch.int32, device=dev)
    kern = ops.prefill_attention_tc if tc else ops.prefill_attention
    fn = lambda: kern(q, kc, vc, work, info, bt, hq, hkv, out)
    name = "prefill_attention_tc" if tc else "prefill_attention"
    if not timed:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return {"kernel": name, "S": S, "chunk": chunk}
    ms = _time(fn)
    flops = S * hq * 128 * 4 * chunk * chunk / 2
    return {"kernel": name, "S": S, "chunk": chunk, "ms": ms, "tflops": flops / ms / 1e9}


def bench_sample(B, V, timed):
    from .. import ops

    dev = torch.device("cuda", 0)
    logits = torch.randn(B, V, device=dev) * 3
    temp = torch.full((B,), 0.7, device=dev)
    topk = torch.full((B,), 40, dtype=torch.int32, device=dev)
    topp = torch.full((B,), 0.9, device=dev)
    rng = torch.arange(B, dtype=torch.int64, device=dev)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    # serving-like repetition penalty: 1500 earlier ids per row (prompt + output), kept as
    # per-slot counts and occurrence lists
    pen = torch.full((B,), 1.15, device=dev)
    counts = torch.zeros(B, V, dtype=torch.int32, device=dev)
    occ = torch.zeros(B, 4096, dtype=torch.int32, device=dev)
    occ_n = torch.zeros(B, dtype=torch.int32, device=dev)
    rows = torch.arange(B, dtype=torch.int32, device=dev).repeat_interleave(1500)
    ops.count_tokens(counts, rows, torch.randint(0, V, (B * 1500,), dtype=torch.int32, device=dev), occ, occ_n)
    fn = lambda: ops.sample(logits, temp, topk, topp, rng, out, rep_penalty=pen, counts=counts, occ=occ, occ_n=occ_n)
    if not timed:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return {"kernel": "sample", "B": B, "V": V}
    ms = _time(fn)
    return {"kernel": "sample", "B": B, "V": V, "ms": ms, "GBps": B * V * 4 / ms / 1e6}


def bench_moe(T, E, d, F, timed, top_k=2):
    """One MoE FFN layer (route, permute, gather, grouped gate/up + SwiGLU,
    grouped down, combine) on T tokens with E experts, single GPU."""
    import types

    from .. import ops
    from ..models.config import ModelConfig
    from ..models.moe import MoE

    dev = torch.device("cuda", 0)
    cfg = ModelConfig(hidden_size=d, intermediate_size=F, num_experts=E, experts_per_token=top_k)
    L = types.SimpleNamespace(
        w_router=(torch.randn(E, d, device=dev) * 0.02).to(torch.bfloat16),
        w_experts_gu=(torch.randn(E, 2 * F, d, device=dev) * 0.02).to(torch.bfloat16),
        w_experts_down=(torch.randn(E, d, F, device=dev) * 0.02).to(torch.bfloat16))
    moe = MoE(cfg, dev)
    moe.configure(T)
    x = torch.randn(T, d, device=dev).to(torch.bfloat16)
    h = torch.zeros(T, d, device=dev, dtype=torch.bfloat16)
    fn = lambda: moe.forward(x, L, h)
    if not timed:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return {"kernel": "moe", "T": T, "E": E}
    ms = _time(fn)
    flops = 2 * T * top_k * 3 * d * F
    wbytes = 3 * E * d * F * 2
    return {"kernel": "moe", "T": T, "E": E, "d": d, "F": F, "ms": ms, "tflops": flops / ms / 1e9,
            "weight_GBps": wbytes / ms / 1e6}


def bench_gemm_q4k(M, N, K, timed):
    """GEMM with GGUF Q4_K weights (dequantized in the mainloop); reports the
    Q4_K bytes streamed per second and the FLOP rate, plus the same GEMM with
    bf16 weights for comparison."""
    from .. import ops
    from ..quantization import quantize_q4_k

    dev = torch.device("cuda", 0)
    w = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
    qw = quantize_q4_k(w)
    x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    fn = lambda: ops.linear(x, qw, out=out)
    if not timed:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return {"kernel": "gemm_q4k", "M": M, "N": N, "K": K}
    ms = _time(fn)
    ms_bf16 = _time(lambda: ops.linear(x, w, out=out))
    saved = ops.Q4K_DEQUANT_MIN_M, ops.Q4K_DEQUANT_MIN_N
    try:  # each path forced: fused dequant-in-mainloop kernel, and dequant pass + bf16 GEMM
        ops.Q4K_DEQUANT_MIN_M = 1 << 30
        ms_fused = _time(fn)
        ops.Q4K_DEQUANT_MIN_M = ops.Q4K_DEQUANT_MIN_N = 0
        ms_deq = _time(fn)
    finally:
        ops.Q4K_DEQUANT_MIN_M, ops.Q4K_DEQUANT_MIN_N = saved
    return {"kernel": "gemm_q4k", "M": M, "N": N, "K": K, "ms": ms, "q4k_GBps": qw.nbytes() / ms / 1e6,
            "tflops": 2 * M * N * K / ms / 1e9, "bf16_weights_ms": ms_bf16, "fused_ms": ms_fused,
            "dequant_then_bf16_ms": ms_deq}


def bench_gemm_issue(M, N, K, units=3):
    """Cycles per 64-wide k slice spent by the 2-SM GEMM's MMA thread under each
    piece of the pipeline protocol (MMA alone is 512), and cycles per
    cta_group::1 MMA by width; read with clock64 on the issuing thread."""
    from .._ext import cuda_ops
    from .. import ops

    dev = torch.device("cuda", 0)
    a = torch.zeros(M, K, device=dev, dtype=torch.bfloat16)
    b = torch.zeros(N, K, device=dev, dtype=torch.bfloat16)
    cyc = torch.zeros(1, dtype=torch.int64, device=dev)
    err = ops.error_buffer(dev)
    rows = []
    for name, mode, ksub, stages, width in [
            ("mma only", 0, 1, 6, 256), ("mma only, N=192", 0, 1, 6, 192), ("mma only, N=128", 0, 1, 6, 128),
            ("+ commit per slice", 1, 1, 6, 256), ("+ completed-barrier wait per slice", 2, 1, 6, 256),
            ("ring, no loads", 3, 1, 6, 256), ("ring + TMA, 1 slice x 6 stages", 4, 1, 6, 256),
            ("ring + TMA, 2 slices x 3 stages", 4, 2, 3, 256), ("ring + TMA, 2 slices x 2 stages", 4, 2, 2, 256)]:
        for _ in range(2):  # the second run is the one read
            cuda_ops().gemm_issue_probe(a, b, mode, ksub, stages, units, width, cyc, err)
        torch.cuda.synchronize()
        rows.append({"variant": name, "cycles_per_slice": int(cyc.item())})
    for n in (64, 128, 256):
        for _ in range(2):
            cuda_ops().mma_rate_probe(n, 2000, cyc, err)
        torch.cuda.synchronize()
        rows.append({"variant": f"cta_group::1 M=128 N={n} K=16", "cycles_per_mma": int(cyc.item())})
    return {"kernel": "gemm_issue", "M": M, "N": N, "K": K, "rows": rows, "errors": ops.check_errors(dev)}


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("what", choices=["gemm", "gemm_q4k", "gemm_issue", "moe", "decode", "prefill", "sample"])
    p.add_argument("dims", nargs="+", type=int)
    p.add_argument("--epi", default="plain", choices=["plain", "bias", "residual", "swiglu"])
    p.add_argument("--time", action="store_true")
    p.add_argument("--cublas", action="store_true", help="gemm: also time torch.nn.functional.linear")
    p.add_argument("--iters", type=int, default=20, help="gemm: timed launches (200 reach the power cap)")
    a = p.parse_args(argv)
    if a.what == "gemm":
        r = bench_gemm(*a.dims[:3], a.epi, a.time, a.cublas, a.iters)
    elif a.what == "gemm_issue":
        r = bench_gemm_issue(*a.dims[:4])
    elif a.what == "gemm_q4k":
        r = bench_gemm_q4k(*a.dims[:3], a.time)
    elif a.what == "moe":
        r = bench_moe(*a.dims[:4], a.time)
    elif a.what == "decode":
        r = bench_decode(*a.dims[:4], a.time)
    elif a.what == "prefill":
        r = bench_prefill(*a.dims[:4], a.time)
    else:
        r = bench_sample(*a.dims[:2], a.time)
    print(json.dumps(r))


if __name__ == "__main__":
    main()
