"""Serving benchmark: output tokens/s of the continuous-batching engine.

``--workload`` picks the model and request shape (see ``WORKLOADS``); the
default, the headline configuration, is
(Qwen2.5-7B architecture, bf16, random N(0, 0.02) weights from seed 0):
256 concurrent requests, prompt lengths uniform in [512, 2048], token ids
uniform over the 152064-entry vocab, 256 output tokens each (EOS ignored),
chunked prefill with a 2048-token step budget, paged KV with 16-token blocks,
sampling with the runtime defaults (T 0.7, top-k 40, top-p 0.9, repetition
penalty 1.15).  One benchmark "step" serves the whole workload to completion.

    python bench.py --gpus N --steps K --warmup W            (torchrun for N > 1)
    python bench.py --impl reference ...                      reference arm

The device-timed value brackets the K steps with CUDA events (barrier +
synchronize on both sides, max over ranks).  The ``e2e`` value serves one more
copy of the workload through the wire API: rank 0 runs the socket server and
LLMBackend (the other ranks follow its steps), and client processes stream
every request with ``KapslClient.infer_stream``; it is timed with the host
clock from the first request sent to the last token received.  Every engine
step copies its inputs host->device from pinned memory and reads its sampled
tokens back device->host.  Weights (15 GB) and the KV working set are far
larger than the 126 MB L2, so no explicit L2 flush is needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "output tok/s on 8×B200 (device-timed, max over ranks); p50 TTFT; p50 TPOT"
REASON_BITS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


# Serving workloads: synthetic uniform-random token ids, random-init weights.
WORKLOADS = {
    # 256 concurrent requests, prompts U[512, 2048], 256 output tokens
    "qwen2.5-7b": dict(model="qwen2.5-7b", num_requests=256, min_prompt=512, max_prompt=2048, output_len=256),
    # 128 requests, 1024-token prompts, 256 output tokens; 8 experts top-2
    "mixtral-8x7b": dict(model="mixtral-8x7b", num_requests=128, min_prompt=1024, max_prompt=1024, output_len=256),
    # 64 requests, 4096-token prompts, 512 output tokens; GGUF Q4_K linear layers
    "llama-3-70b-q4k": dict(model="llama-3-70b-q4k", num_requests=64, min_prompt=4096, max_prompt=4096,
                            output_len=512),
}
# CPU backend served over a Unix socket (KapslClient.infer_stream), f32 GGUF tiny Llama:
# 4 requests of 128 token ids, greedy 64 output tokens (no GPU)
WORKLOADS["tiny-llama-cpu"] = dict(model="tiny-llama", num_requests=4, min_prompt=128, max_prompt=128, output_len=64)
# disaggregated prefill/decode (``--parallel pd``): 32 requests, 8192-token prompts, 128 output tokens
WORKLOADS["llama-3-8b-pd"] = dict(model="llama-3-8b", num_requests=32, min_prompt=8192, max_prompt=8192,
                                  output_len=128)
# The in-repo library baseline (B1: cuBLAS + NCCL + vLLM flash-attention on the same engine,
# `bench.py --impl b1`) for the headline workload, output tok/s by GPU count, as recorded in
# BASELINE.md; vs_baseline = value / this (null where B1 has no number for that count).
B1_TOK_S = {("qwen2.5-7b", 1): 4351.21}

MODEL_LABEL = {"qwen2.5-7b": "Qwen2.5-7B-arch", "mixtral-8x7b": "Mixtral-8x7B-arch",
               "llama-3-70b-q4k": "Llama-3-70B-arch Q4_K", "llama-3-8b": "Llama-3-8B-arch"}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="kapsl", choices=["kapsl", "reference", "b1"],
                   help="kapsl: this framework; reference: the reference's own build; b1: the in-repo library "
                        "baseline (cuBLAS via torch, NCCL all-reduce, vLLM flash-attention, torch sampling) on the "
                        "same engine")
    p.add_argument("--workload", default="qwen2.5-7b", choices=sorted(WORKLOADS),
                   help="named serving workload (model + request shape); the flags below override it")
    p.add_argument("--model", default=None)
    p.add_argument("--num-requests", type=int, default=None)
    p.add_argument("--min-prompt", type=int, default=None)
    p.add_argument("--max-prompt", type=int, default=None)
    p.add_argument("--output-len", type=int, default=None)
    p.add_argument("--chunk", type=int, default=2048)
    p.add_argument("--parallel", default="tp", choices=["dp", "tp", "pd", "pp"],
                   help="tp: one model over all N GPUs (the named TP=N config, strong scaling); "
                        "dp: N independent replicas, each serving its own copy of the workload; "
                        "pd: disaggregated, prefill on GPUs [0, N/2) and decode on [N/2, N), TP N/2 each; "
                        "pp: N pipeline stages (layers split over the GPUs, hidden states over NCCL "
                        "point-to-point, two micro-batches per step)")
    p.add_argument("--kv-mode", default="p2p", choices=["p2p", "copy"],
                   help="pd: KV transfer by the P2P push kernel or the copy-engine baseline")
    p.add_argument("--tp-mode", default="fused", choices=["fused", "nccl"],
                   help="row-parallel reduction: fused NVLink kernels or the NCCL baseline")
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--no-overlap", action="store_true",
                   help="one engine step at a time (the host waits for each step's tokens before the next launch)")
    p.add_argument("--num-layers", type=int, default=0, help="override (testing only; invalid for the metric)")
    p.add_argument("--warmup-scale", type=float, default=1.0,
                   help="fraction of requests served by each warm-up step")
    p.add_argument("--no-e2e", action="store_true",
                   help="skip the end-to-end pass through the serving API (secondary workloads; the headline "
                        "line always carries it)")
    p.add_argument("--profile", action="store_true",
                   help="per-step host/device breakdown of the timed region (stderr, one JSON line per rank)")
    a = p.parse_args()
    for k, v in WORKLOADS[a.workload].items():
        if getattr(a, k) is None:
            setattr(a, k, v)
    return a


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        try:
            for line in open(self.path):
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 4:
                    continue
                try:
                    sm.append(float(parts[0]))
                    mx = max(mx, float(parts[1]))
                    bits = int(parts[3], 16) if parts[3].startswith("0x") else int(parts[3])
                except ValueError:
                    continue
                for b, name in REASON_BITS.items():
                    if bits & b and name != "gpu_idle":
                        reasons.add(name)
        except OSError:
            pass
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_workload(args, vocab: int, seed: int = 1):
    import numpy as np

    rng = np.random.default_rng(seed)
    lens = rng.integers(args.min_prompt, args.max_prompt + 1, size=args.num_requests)
    return [rng.integers(0, vocab, size=int(n)).tolist() for n in lens]


def reference_arm(args):
    """The reference is a Rust/maturin project; it cannot be installed offline here."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    why = ("reference (kapsl-sdk, Rust crates + PyO3/maturin) is not installable offline: pip reports "
           "BackendUnavailable 'No module named maturin' and no cargo/rustc toolchain exists; its LLM path "
           "also needs ONNX Runtime binaries downloaded at build time")
    if os.path.isdir(ref_dir) and any(n.startswith("kapsl_sdk") for n in os.listdir(ref_dir)):
        why = "reference kapsl_sdk installed but it is a client only: no runtime server binary to serve the workload"
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}))
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    if args.workload == "tiny-llama-cpu":
        return run_cpu_serving(args)

    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)

    from kapsl_sdk_b200._ext import cuda_ops
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.config import get_preset

    cuda_ops()
    if args.profile:
        os.environ["KAPSL_LLM_PROFILE"] = "1"
    if args.parallel == "pd":
        return run_pd(args, dev, world, rank, local)
    cfg = get_preset(args.model)
    if args.num_layers:
        cfg.num_layers = args.num_layers
    tp_comm = None
    if args.parallel == "tp" and world > 1:
        from kapsl_sdk_b200.parallel.tp import TPComm

        tp_comm = TPComm.from_world(mode="nccl" if args.impl == "b1" else args.tp_mode)
    pp_stage = None
    if args.parallel == "pp" and world > 1:
        from kapsl_sdk_b200.parallel.pp import PipelineStage

        pp_stage = PipelineStage(rank, world, cfg.num_layers, micro_batches=2)
        args.no_e2e = True  # the serving front end drives tensor-parallel groups, not pipeline stages
    model_cls = None
    if args.impl == "b1":
        from kapsl_sdk_b200.models.baseline import BaselineCausalLM as model_cls
    ecfg = EngineConfig(max_num_seqs=args.num_requests, max_num_batched_tokens=args.chunk,
                        max_model_len=args.max_prompt + args.output_len + 16, use_cuda_graph=not args.no_graph,
                        overlap_steps=not args.no_overlap)
    engine = LLMEngine(cfg, device=dev, engine_cfg=ecfg, tp_comm=tp_comm, seed=0, model_cls=model_cls,
                       pp_stage=pp_stage)
    shared = tp_comm is not None or pp_stage is not None  # one workload over all ranks
    weight_gb = (torch.cuda.memory_allocated(dev) - engine.pool.storage.numel() * engine.pool.storage.element_size()) / 1e9
    # data-parallel replicas serve their own copy of the workload (weak scaling);
    # tensor parallel shares one workload across the ranks (strong scaling).
    # A fresh prompt set for every pass (warm-up, timed, end-to-end), so no pass
    # can reuse KV blocks that an earlier pass left in the prefix cache.
    rank_seed = 1000 * (0 if shared else rank)

    def prompts_for(pass_idx: int):
        return make_workload(args, cfg.vocab_size, seed=1 + rank_seed + pass_idx)
    params = SamplingParams(max_new_tokens=args.output_len, temperature=0.7, top_k=40, top_p=0.9,
                            repetition_penalty=1.15, ignore_eos=True)

    def barrier():
        if world > 1:
            dist.barrier()

    def serve(ps):
        seqs = [engine.add_request(f"bench-{serve.n}-{i}", p, params) for i, p in enumerate(ps)]
        serve.n += 1
        while engine.has_unfinished():
            engine.step()
        return seqs

    serve.n = 0
    nwarm = max(1, int(args.num_requests * args.warmup_scale))
    npass = 0
    for _ in range(args.warmup):
        serve(prompts_for(npass)[:nwarm])
        npass += 1
    torch.cuda.synchronize()
    barrier()

    # ---------------- device-timed region
    if engine.profile is not None:
        for k in list(engine.profile):
            engine.profile[k] = 0
        if os.environ.get("KAPSL_TRACE_DIR"):
            engine.profile["trace"] = []
        if tp_comm is not None and hasattr(tp_comm, "phase_times"):
            tp_comm.phase_times(reset=True)
    wall0 = time.perf_counter()
    launches0 = engine.runner.launches
    h2d0, d2h0 = engine.runner.stats["h2d_bytes"], engine.runner.stats["d2h_bytes"]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    all_seqs = []
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        timed_prompts = [prompts_for(npass + i) for i in range(args.steps)]
        start.record()
        for i in range(args.steps):
            all_seqs.extend(serve(timed_prompts[i]))
        end.record()
        torch.cuda.synchronize()
        barrier()
    ms = start.elapsed_time(end)
    if engine.profile is not None:
        trace = engine.profile.pop("trace", None)
        if trace is not None:
            with open(os.path.join(os.environ["KAPSL_TRACE_DIR"], f"trace_n{world}_r{rank}.json"), "w") as f:
                json.dump(trace, f)
        prof = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in engine.profile.items()}
        prof.update(rank=rank, wall_s=round(time.perf_counter() - wall0, 3), device_ms=round(ms, 1))
        if tp_comm is not None and hasattr(tp_comm, "phase_times"):
            prof["tp_reduce"] = {k: round(v, 2) for k, v in tp_comm.phase_times().items()}
        print(json.dumps({"profile": prof}), file=sys.stderr, flush=True)
    launches = engine.runner.launches - launches0
    h2d = (engine.runner.stats["h2d_bytes"] - h2d0) / args.steps
    d2h = (engine.runner.stats["d2h_bytes"] - d2h0) / args.steps
    out_tokens = sum(len(s.output_ids) for s in all_seqs)
    ttft = statistics.median([s.ttft() for s in all_seqs if s.ttft() is not None])
    tpot = statistics.median([s.tpot() for s in all_seqs if s.tpot() is not None])

    # ---------------- end to end through the serving API (host clock)
    barrier()
    e2e_prompts = prompts_for(npass + args.steps)
    h2d1, d2h1 = engine.runner.stats["h2d_bytes"], engine.runner.stats["d2h_bytes"]
    group = tp_comm is not None and world > 1  # data-parallel replicas each serve their own copy
    if args.no_e2e:
        e2e_tokens, e2e_s = 0, 1.0
    else:
        e2e_tokens, e2e_s = serve_e2e(engine, world if group else 1, rank if group else 0, params, e2e_prompts)
    e2e_h2d = engine.runner.stats["h2d_bytes"] - h2d1
    e2e_d2h = engine.runner.stats["d2h_bytes"] - d2h1
    barrier()

    # correctness of the timed pass: ranks that share one workload (tensor / pipeline
    # parallel) must have produced the same tokens; every token id lies in the vocabulary
    digest = outputs_digest(all_seqs)
    in_vocab = all(0 <= t < cfg.vocab_size for s in all_seqs for t in s.output_ids)
    vals = torch.tensor([ms, out_tokens, e2e_s, e2e_tokens, ttft, tpot], dtype=torch.float64, device=dev)
    checks = torch.tensor([digest, int(in_vocab)], dtype=torch.int64, device=dev)
    if world > 1:
        gathered = [torch.zeros_like(vals) for _ in range(world)]
        dist.all_gather(gathered, vals)
        g = torch.stack(gathered)
        ms_max = float(g[:, 0].max())
        e2e_max = float(g[:, 2].max())
        if not shared:
            tot_tokens = float(g[:, 1].sum())
            tot_e2e_tokens = float(g[:, 3].sum())
        else:
            tot_tokens = float(g[0, 1])
            tot_e2e_tokens = float(g[0, 3])  # served by rank 0
        e2e_max = float(g[0, 2]) if shared else e2e_max
        ttft_all = float(g[:, 4].max())
        tpot_all = float(g[:, 5].max())
        gc = [torch.zeros_like(checks) for _ in range(world)]
        dist.all_gather(gc, checks)
        gc = torch.stack(gc)
        ranks_agree = bool((gc[:, 0] == gc[0, 0]).all()) if shared else None
        in_vocab = bool(gc[:, 1].all())
    else:
        ranks_agree = None
        ms_max, e2e_max, tot_tokens, tot_e2e_tokens, ttft_all, tpot_all = ms, e2e_s, out_tokens, e2e_tokens, ttft, tpot
    value = tot_tokens / (ms_max / 1000.0)
    par = ((f"tp{world}" + ("" if world == 1 else f"-{args.tp_mode}")) if args.parallel == "tp"
           else f"{args.parallel}{world}")
    if args.impl == "b1":
        par += " (library baseline: cuBLAS + NCCL + vLLM flash-attention)"
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "output tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3),
            "higher_is_better": True, "scaling": "strong" if shared or args.parallel == "tp" else "weak",
            "vs_baseline": (round(value / B1_TOK_S[(args.model, world)], 3)
                            if args.impl == "kapsl" and args.parallel == "tp" and (args.model, world) in B1_TOK_S
                            and args.num_requests == WORKLOADS["qwen2.5-7b"]["num_requests"] else None),
            "dtype": "bf16", "data": "synthetic token ids, random-init weights N(0,0.02) seed 0",
            "config": {"model": MODEL_LABEL.get(args.model, args.model),
                       "global_batch": args.num_requests * (1 if shared else world),
                       "seq_len": f"prompt U[{args.min_prompt},{args.max_prompt}] + {args.output_len} out",
                       "parallelism": par, "chunked_prefill": args.chunk, "kv_block": 16,
                       "l2": f"inputs larger than L2 ({weight_gb:.0f} GB weights, GB-scale KV), no flush",
                       "num_layers": cfg.num_layers},
            "p50_ttft_ms": round(ttft_all * 1000, 2), "p50_tpot_ms": round(tpot_all * 1000, 3),
            "clocks": clocks.summary(),
            "e2e": None if args.no_e2e else {"value": round(tot_e2e_tokens / e2e_max, 2), "unit": "output tokens/s",
                    "h2d_bytes_per_step": int(e2e_h2d), "d2h_bytes_per_step": int(e2e_d2h),
                    "api": "KapslClient.infer_stream over a Unix socket (token-id prompts; rank 0 serves, "
                           "other ranks follow its steps)",
                    "timing": "host clock, first request sent to last token received, client processes"},
            "gpu_launches": int(launches),
            "check": {"tokens_in_vocab": in_vocab, "ranks_agree": ranks_agree,
                      "what": "timed pass: every output id inside the vocabulary; ranks sharing one workload "
                              "produced identical outputs (digest over all sequences)"},
        }
        if args.impl == "b1":
            line["impl"] = "b1-library-baseline"
        print(json.dumps(line))
    engine.shutdown()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def outputs_digest(seqs) -> int:
    """63-bit digest of every sequence's output ids, in request order."""
    import hashlib

    h = hashlib.sha1()
    for s in seqs:
        h.update(len(s.output_ids).to_bytes(4, "little"))
        for t in s.output_ids:
            h.update(int(t).to_bytes(4, "little", signed=True))
    return int.from_bytes(h.digest()[:8], "little") & ((1 << 63) - 1)


def _e2e_client(sock: str, prompts: list, go, q) -> None:
    """One client process: a thread per prompt streams it through KapslClient;
    reports (tokens received, time of the first send, time of the last token)."""
    import threading

    import numpy as np

    from kapsl_sdk import KapslClient

    got = [0] * len(prompts)

    def run(i):
        c = KapslClient(sock)
        data = np.asarray(prompts[i], dtype=np.int32).tobytes()
        n = 0
        for _ in c.infer_stream(0, [1, len(prompts[i])], "int32", data):
            n += 1
        got[i] = n

    th = [threading.Thread(target=run, args=(i,)) for i in range(len(prompts))]
    go.wait()
    t0 = time.monotonic()
    for t in th:
        t.start()
    for t in th:
        t.join()
    q.put((sum(got), t0, time.monotonic()))


def serve_e2e(engine, world: int, rank: int, params, prompts: list, nclients: int = 4):
    """Serve ``prompts`` through the wire API: rank 0 runs KapslServer + LLMBackend
    (over a GroupLeader when world > 1, the other ranks follow its steps) on a
    Unix socket, and ``nclients`` client processes stream every prompt
    concurrently with KapslClient.infer_stream.  Returns (tokens, seconds) on
    rank 0, (0, 0) elsewhere."""
    import multiprocessing as mp
    import threading

    from kapsl_sdk_b200.llm.backend import LLMBackend, RuntimeConfig
    from kapsl_sdk_b200.parallel.group import GroupLeader, StepChannel, follow
    from kapsl_sdk_b200.server import KapslServer

    chan = None
    if world > 1:
        import torch.distributed as dist

        name = [f"kapsl-bench-{os.getpid()}-{os.urandom(3).hex()}" if rank == 0 else None]
        dist.broadcast_object_list(name, src=0)
        chan = StepChannel(name[0], world, rank)
        dist.barrier()
        if rank != 0:
            follow(engine, chan)
            chan.close()
            return 0, 0.0
    eng = GroupLeader(engine, chan) if chan is not None else engine
    backend = LLMBackend(eng, runtime_config=RuntimeConfig(sampling=params), own_thread=False)
    tmp = tempfile.mkdtemp(prefix="kapsl-e2e-")
    sock = os.path.join(tmp, "kapsl.sock")
    srv = KapslServer({0: backend}).listen_unix(sock).start()
    ctx = mp.get_context("spawn")
    go, q = ctx.Event(), ctx.Queue()
    procs = [ctx.Process(target=_e2e_client, args=(sock, prompts[i::nclients], go, q), daemon=True)
             for i in range(nclients)]
    for p in procs:
        p.start()
    results = []

    def watch():
        for _ in procs:
            results.append(q.get())
        backend._stop.set()

    threading.Thread(target=watch, daemon=True).start()
    time.sleep(3.0)  # client processes import and connect before the start signal
    go.set()
    try:
        backend.run()
    finally:
        srv.stop()
        for p in procs:
            p.join(30)
        if chan is not None:
            eng.stop_followers()
            chan.close()
    tokens = sum(r[0] for r in results)
    secs = max(r[2] for r in results) - min(r[1] for r in results)
    return tokens, secs


def _cpu_server(gguf: str, sock: str, num_requests: int, chunk: int, max_len: int, output_len: int) -> None:
    """Server process of the CPU workload: GGUF -> CPU engine -> LLMBackend -> socket server."""
    from kapsl_sdk_b200.llm.backend import LLMBackend, RuntimeConfig
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.loaders.gguf import load_gguf_model
    from kapsl_sdk_b200.server import KapslServer

    cfg, model, tok = load_gguf_model(gguf, "cpu")
    engine = LLMEngine(cfg, weights=model, device="cpu",
                       engine_cfg=EngineConfig(max_num_seqs=num_requests, max_num_batched_tokens=chunk,
                                               max_model_len=max_len, block_size=16, num_blocks=num_requests * 16),
                       seed=0)
    rc = RuntimeConfig(sampling=SamplingParams.greedy(output_len, ignore_eos=True))
    backend = LLMBackend(engine, tokenizer=tok, runtime_config=rc, own_thread=False)
    srv = KapslServer(models={0: backend}).listen_unix(sock).start()
    backend.run()  # the engine loop on the thread that built the model (one OpenMP team)
    srv.stop()


def run_cpu_serving(args) -> int:
    """Tiny Llama f32 GGUF on the CPU backend behind the socket server (its own
    process), driven by concurrent KapslClient.infer_stream calls with
    token-id prompts.  Host-timed on the client side (there is no device); a
    step serves all requests to completion."""
    import multiprocessing as mp
    import threading

    import numpy as np
    import torch

    from kapsl_sdk import KapslClient
    from kapsl_sdk_b200.loaders.gguf import write_gguf_model
    from kapsl_sdk_b200.models.config import get_preset
    from kapsl_sdk_b200.models.llama import random_full_weights

    cfg = get_preset(args.model)
    tmp = tempfile.mkdtemp(prefix="kapsl-bench-")
    gguf = os.path.join(tmp, "tiny-llama-f32.gguf")
    write_gguf_model(gguf, cfg, random_full_weights(cfg, torch.device("cpu"), seed=0, std=0.02), quant="f32")
    sock = os.path.join(tmp, "kapsl.sock")
    proc = mp.get_context("spawn").Process(target=_cpu_server, daemon=True, args=(
        gguf, sock, args.num_requests, args.chunk, args.max_prompt + args.output_len + 16, args.output_len))
    proc.start()
    t_wait = time.perf_counter()
    while not os.path.exists(sock):
        if not proc.is_alive() or time.perf_counter() - t_wait > 300:
            raise SystemExit(f"CPU server did not come up (exit code {proc.exitcode})")
        time.sleep(0.1)

    def one_pass(seed: int):
        prompts = make_workload(args, cfg.vocab_size, seed=seed)
        stats = [None] * len(prompts)

        def run(i):
            c = KapslClient(sock)
            data = np.asarray(prompts[i], dtype=np.int32).tobytes()
            t0 = time.perf_counter()
            times = []
            for _ in c.infer_stream(0, [1, len(prompts[i])], "int32", data):
                times.append(time.perf_counter())
            stats[i] = (t0, times)

        th = [threading.Thread(target=run, args=(i,)) for i in range(len(prompts))]
        t0 = time.perf_counter()
        for t in th:
            t.start()
        for t in th:
            t.join()
        return time.perf_counter() - t0, stats

    try:
        for i in range(args.warmup):
            one_pass(1000 + i)
        walls, all_stats = [], []
        for i in range(args.steps):
            w, st = one_pass(1 + i)  # the first timed pass uses the workload's seed 1
            walls.append(w)
            all_stats.extend(st)
    finally:
        proc.terminate()
        proc.join(10)
    tokens = sum(len(t) for _, t in all_stats)
    wall = sum(walls)
    ttft = statistics.median([t[0] - t0 for t0, t in all_stats])
    tpot = statistics.median([(t[-1] - t[0]) / (len(t) - 1) for _, t in all_stats if len(t) > 1])
    print(json.dumps({
        "metric": METRIC, "value": round(tokens / wall, 2), "unit": "output tokens/s", "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1000, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic token ids (seed 1), random-init weights N(0,0.02) seed 0, f32 GGUF",
        "config": {"model": "tiny-Llama (4 layers, d 512, 8/8 heads of 64, FFN 1408, vocab 32000)",
                   "global_batch": args.num_requests, "seq_len": f"{args.max_prompt} prompt + {args.output_len} out",
                   "parallelism": "cpu", "kv_block": 16, "timing": "host clock, client side",
                   "api": "KapslClient.infer_stream over a Unix socket (token-id prompts), server in its own process"},
        "p50_ttft_ms": round(ttft * 1000, 2), "p50_tpot_ms": round(tpot * 1000, 3),
        "e2e": {"value": round(tokens / wall, 2), "unit": "output tokens/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0, "api": "KapslClient.infer_stream"},
        "gpu_launches": 0}))
    return 0


def run_pd(args, dev, world: int, rank: int, local: int) -> int:
    """Disaggregated prefill/decode through the KV connector; device-timed over
    whole serving passes (barrier + synchronize on both sides, max over ranks)."""
    import torch
    import torch.distributed as dist

    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.config import get_preset
    from kapsl_sdk_b200.parallel.disagg import Disaggregated
    from kapsl_sdk_b200.parallel.tp import TPComm

    if world < 2:
        raise SystemExit("--parallel pd needs at least 2 GPUs")
    cfg = get_preset(args.model)
    if args.num_layers:
        cfg.num_layers = args.num_layers

    def make(role, group, gi, n):
        tp = TPComm(n, gi, dev, args.tp_mode, group=group) if n > 1 else None
        ecfg = EngineConfig(max_num_seqs=args.num_requests, max_num_batched_tokens=args.chunk,
                            max_model_len=args.max_prompt + args.output_len + 16, use_cuda_graph=not args.no_graph,
                            shareable_kv=(role == "decode"))
        return LLMEngine(cfg, device=dev, engine_cfg=ecfg, tp_comm=tp, seed=0)

    d = Disaggregated(make, mode=args.kv_mode)
    params = SamplingParams(max_new_tokens=args.output_len, temperature=0.7, top_k=40, top_p=0.9,
                            repetition_penalty=1.15, ignore_eos=True)
    nwarm = max(1, int(args.num_requests * args.warmup_scale))
    for i in range(args.warmup):
        d.serve(make_workload(args, cfg.vocab_size, seed=1 + i)[:nwarm], params)
    torch.cuda.synchronize()
    dist.barrier()
    launches0 = d.engine.runner.launches
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    seqs = []
    with ClockSampler(local) as clocks:
        dist.barrier()
        torch.cuda.synchronize()
        batches = [make_workload(args, cfg.vocab_size, seed=100 + i) for i in range(args.steps)]
        start.record()
        for b in batches:
            _, s = d.serve(b, params)
            seqs.extend(s or [])
        end.record()
        torch.cuda.synchronize()
        dist.barrier()
    ms = start.elapsed_time(end)
    out_tokens = sum(len(s.output_ids) for s in seqs)
    ttft = statistics.median([s.ttft() for s in seqs]) if seqs else 0.0
    tpot = statistics.median([s.tpot() for s in seqs if s.tpot() is not None]) if seqs else 0.0
    vals = torch.tensor([ms, out_tokens, ttft, tpot, d.engine.runner.launches - launches0], dtype=torch.float64,
                        device=dev)
    g = [torch.zeros_like(vals) for _ in range(world)]
    dist.all_gather(g, vals)
    g = torch.stack(g)
    P = world // 2
    ms_max = float(g[:, 0].max())
    tokens = float(g[P, 1])
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(tokens / (ms_max / 1000.0), 2), "unit": "output tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic token ids, random-init weights N(0,0.02) seed 0",
            "config": {"model": MODEL_LABEL.get(args.model, args.model), "global_batch": args.num_requests,
                       "seq_len": f"prompt U[{args.min_prompt},{args.max_prompt}] + {args.output_len} out",
                       "parallelism": f"pd: prefill tp{P} + decode tp{P}, kv {args.kv_mode}",
                       "chunked_prefill": args.chunk, "kv_block": 16,
                       "l2": "inputs larger than L2 (GB-scale weights and KV), no flush"},
            "p50_ttft_ms": round(float(g[P, 2]) * 1000, 2), "p50_tpot_ms": round(float(g[P, 3]) * 1000, 3),
            "clocks": clocks.summary(), "gpu_launches": int(g[:, 4].sum())}))
    d.close()
    d.engine.shutdown()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
