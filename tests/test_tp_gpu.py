"""Tensor and expert parallelism on 2, 4 or 8 GPUs (skipped with fewer): the
fused NVLink row-parallel reduction against the NCCL baseline and against
TP1 (with padded query heads at 8 ranks), and an expert-parallel MoE model
against one GPU, driven as child processes (one per GPU) over NCCL with NVLS off."""
import json
import os
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = textwrap.dedent(r"""
import json, os, sys, torch
from datetime import timedelta
import torch.distributed as dist
sys.path.insert(0, os.environ["KAPSL_ROOT"])
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
from kapsl_sdk_b200 import ops
from kapsl_sdk_b200.parallel.tp import TPComm
from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
from kapsl_sdk_b200.llm.sequence import SamplingParams
from kapsl_sdk_b200.models.config import ModelConfig
dev = torch.device("cuda", rank)
out = {}
# 1) fused row-parallel reduction vs a dense reference
torch.manual_seed(0)
T, K, N = 300, 1024, 512
x_full = torch.randn(T, K * world, device=dev, dtype=torch.bfloat16)
w_full = torch.randn(N, K * world, device=dev, dtype=torch.bfloat16) / 50
h0 = torch.randn(T, N, device=dev, dtype=torch.bfloat16)
ref = h0.float() + x_full.float() @ w_full.float().T
xs, ws = x_full[:, rank * K:(rank + 1) * K].contiguous(), w_full[:, rank * K:(rank + 1) * K].contiguous()
for mode in ("fused", "nccl"):
    tp = TPComm(world, rank, dev, mode, max_tokens=512, hidden=N)
    h = tp.residual_stream(T) if mode == "fused" else torch.empty_like(h0)
    h.copy_(h0)
    for _ in range(3):  # repeated use exercises the epoch barriers
        h.copy_(h0)
        tp.row_parallel_residual(xs, ws, h)
    torch.cuda.synchronize()
    out[mode] = float((h.float() - ref).abs().max())
    out[mode + "_err"] = ops.check_errors(dev)
    tp.close()
    if mode == "fused":
        # reduction + residual + RMSNorm: flag-carrying-line kernel one-shot (every row on
        # every rank) and two-shot (owned rows + all-gather of the normed rows), and the
        # barrier + pull kernel; all sum in rank order, so their rows agree bit for bit
        nw = (torch.rand(N, device=dev) + 0.5).to(torch.bfloat16)
        hb = ref.to(torch.bfloat16).float()
        xref = hb * torch.rsqrt(hb.pow(2).mean(-1, keepdim=True) + 1e-6) * nw.float()
        rpr = (T + world - 1) // world
        own = slice(rank * rpr, min(T, (rank + 1) * rpr))
        xs_by = {}
        for var in ("pull", "ll1", "ll2"):
            tp = TPComm(world, rank, dev, "fused", max_tokens=512, hidden=N)
            tp.ll1_rows, tp.ll2_rows = (512, 0) if var == "ll1" else (0, 512)
            tp.norm_kernel = "pull" if var == "pull" else "ll"
            tp.close()
            tp._setup_symmetric(512, N)
            h = tp.residual_stream(T)
            for _ in range(3):  # repeated calls exercise the epochs, flags and one-shot slot parity
                h.copy_(h0)
                xn = tp.row_parallel_norm(xs, ws, h, nw, 1e-6)
            torch.cuda.synchronize()
            rows = slice(0, T) if var == "ll1" else own
            out["norm_h_" + var] = float((h[rows].float() - ref[rows]).abs().max())
            out["norm_x_" + var] = float((xn.float() - xref).abs().max())
            out["norm_err_" + var] = ops.check_errors(dev)
            xs_by[var] = xn.clone()
            tp.close()
        out["norm_bitwise"] = all(torch.equal(xs_by["pull"], xs_by[v]) for v in ("ll1", "ll2"))
        # large batches: the scatter GEMM (rows pushed to their owners from the epilogue,
        # local reduction) against the pull reduction, bit for bit, and against fp32
        T2, K2, N2 = 2048, 512, 2048
        x2 = torch.randn(T2, K2 * world, device=dev, dtype=torch.bfloat16)
        w2 = torch.randn(N2, K2 * world, device=dev, dtype=torch.bfloat16) / 40
        h2 = torch.randn(T2, N2, device=dev, dtype=torch.bfloat16)
        nw2 = (torch.rand(N2, device=dev) + 0.5).to(torch.bfloat16)
        ref2 = (h2.float() + x2.float() @ w2.float().T).to(torch.bfloat16).float()
        xref2 = ref2 * torch.rsqrt(ref2.pow(2).mean(-1, keepdim=True) + 1e-6) * nw2.float()
        xs2 = x2[:, rank * K2:(rank + 1) * K2].contiguous()
        ws2 = w2[:, rank * K2:(rank + 1) * K2].contiguous()
        big = {}
        for var in ("pull", "scatter"):
            tp = TPComm(world, rank, dev, "fused", max_tokens=T2, hidden=N2)
            tp.large_kernel = var
            hh = tp.residual_stream(T2)
            for _ in range(2):
                hh.copy_(h2)
                xn = tp.row_parallel_norm(xs2, ws2, hh, nw2, 1e-6)
            torch.cuda.synchronize()
            out["large_used_" + var] = tp._scatter_ok(xs2, ws2)
            out["large_x_" + var] = float((xn.float() - xref2).abs().max())
            out["large_err_" + var] = ops.check_errors(dev)
            big[var] = xn.clone()
            tp.close()
        out["large_bitwise"] = bool(torch.equal(big["pull"], big["scatter"]))
# 2) a small model: TP=world greedy tokens vs TP=1 on rank 0
# 12 query heads over 2 KV heads: at 8 ranks each KV group of 6 is padded to 8 query heads
cfg = ModelConfig(name="s", arch="qwen2", vocab_size=1024, hidden_size=512, intermediate_size=1024, num_layers=2,
                  num_heads=12, num_kv_heads=2, head_dim=128, max_position=1024, qkv_bias=True,
                  bos_token_id=None, eos_token_id=None)
prompts = [[(i * 37 + j) % 1000 for j in range(n)] for i, n in enumerate((40, 130, 7))]
tp = TPComm(world, rank, dev, "fused")
eng = LLMEngine(cfg, device=dev, engine_cfg=EngineConfig(max_num_seqs=8, max_num_batched_tokens=128,
                max_model_len=512, num_blocks=256), tp_comm=tp, seed=0)
toks = eng.generate(prompts, SamplingParams.greedy(12, ignore_eos=True))
out["tp_tokens"] = toks
out["engine_err"] = ops.check_errors(dev)
eng.shutdown()
tp.close()
tp = TPComm(world, rank, dev, "nccl")
eng = LLMEngine(cfg, device=dev, engine_cfg=EngineConfig(max_num_seqs=8, max_num_batched_tokens=128,
                max_model_len=512, num_blocks=256), tp_comm=tp, seed=0)
out["nccl_tokens"] = eng.generate(prompts, SamplingParams.greedy(12, ignore_eos=True))
eng.shutdown()
tp.close()
if rank == 0:
    e1 = LLMEngine(cfg, device=dev, engine_cfg=EngineConfig(max_num_seqs=8, max_num_batched_tokens=128,
                   max_model_len=512, num_blocks=256), seed=0)
    out["tp1_tokens"] = e1.generate(prompts, SamplingParams.greedy(12, ignore_eos=True))
# 3) mixture of experts: experts split over the ranks (fused peer-pull combine) vs one GPU
mcfg = ModelConfig(name="m", arch="mixtral", vocab_size=1024, hidden_size=512, intermediate_size=512, num_layers=2,
                   num_heads=8, num_kv_heads=8, head_dim=128, max_position=1024, num_experts=8,
                   experts_per_token=2, bos_token_id=None, eos_token_id=None)
tp = TPComm(world, rank, dev, "fused")
eng = LLMEngine(mcfg, device=dev, engine_cfg=EngineConfig(max_num_seqs=8, max_num_batched_tokens=128,
                max_model_len=512, num_blocks=256), tp_comm=tp, seed=0)
out["ep_tokens"] = eng.generate(prompts, SamplingParams.greedy(12, ignore_eos=True))
out["ep_err"] = ops.check_errors(dev)
eng.shutdown()
tp.close()
if rank == 0:
    e1 = LLMEngine(mcfg, device=dev, engine_cfg=EngineConfig(max_num_seqs=8, max_num_batched_tokens=128,
                   max_model_len=512, num_blocks=256), seed=0)
    out["ep1_tokens"] = e1.generate(prompts, SamplingParams.greedy(12, ignore_eos=True))
print("RESULT " + json.dumps(out), flush=True)
dist.barrier()
dist.destroy_process_group()
""")


def _run(world):
    env = dict(os.environ, KAPSL_ROOT=ROOT, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1", MASTER_PORT="29561",
               WORLD_SIZE=str(world))
    procs = []
    for r in range(world):
        procs.append(subprocess.Popen([sys.executable, "-c", WORKER], env=dict(env, RANK=str(r), LOCAL_RANK=str(r)),
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            o, _ = p.communicate(timeout=600)
        except subprocess.TimeoutExpired:
            p.kill()
            o, _ = p.communicate()
        outs.append((p.returncode, o))
    return outs


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tensor_and_expert_parallel():
    world = 1 << (min(torch.cuda.device_count(), 8).bit_length() - 1)  # 2, 4 or 8 ranks
    outs = _run(world)
    res = []
    for rc, o in outs:
        line = [l for l in o.splitlines() if l.startswith("RESULT ")]
        assert rc == 0 and line, o[-3000:]
        res.append(json.loads(line[0][7:]))
    for r in res:
        assert r["fused_err"] == 0 and r["nccl_err"] == 0 and r["engine_err"] == 0 and r["ep_err"] == 0
        # outputs of magnitude ~3: bf16 rounding of each partial and of the sum is ~0.01 each;
        # NCCL's bf16 ring rounds once per hop, so its error grows with the rank count
        assert r["fused"] < 0.05 and r["nccl"] < 0.025 * world, r
        bad = [v for v in ("pull", "ll1", "ll2")
               if not (r["norm_err_" + v] == 0 and r["norm_h_" + v] < 0.05 and r["norm_x_" + v] < 0.05)]
        assert not bad, (bad, r)
        assert r["norm_bitwise"], r
        assert r["large_used_scatter"] and not r["large_used_pull"], r
        assert r["large_err_pull"] == 0 and r["large_err_scatter"] == 0, r
        assert r["large_x_pull"] < 0.05 and r["large_x_scatter"] < 0.05 and r["large_bitwise"], r
    for key in ("tp_tokens", "ep_tokens", "nccl_tokens"):
        assert all(r[key] == res[0][key] for r in res)  # ranks stay in lock step
    # greedy tokens: the reductions round differently (NCCL sums bf16 partials in its own
    # order), so a near-tie can flip a token and the rest of its sequence; top-2 expert
    # routing turns such a flip into a different expert pair, hence the looser MoE bar
    for key, ref, frac in (("tp_tokens", "tp1_tokens", 0.9), ("ep_tokens", "ep1_tokens", 0.8),
                           ("tp_tokens", "nccl_tokens", 0.9)):
        same = sum(a == b for x, y in zip(res[0][key], res[0][ref]) for a, b in zip(x, y))
        assert same >= frac * sum(len(x) for x in res[0][ref]), (key, ref, res[0][key], res[0][ref])
        assert [x[0] for x in res[0][key]] == [y[0] for y in res[0][ref]], (key, ref)  # first tokens exact
