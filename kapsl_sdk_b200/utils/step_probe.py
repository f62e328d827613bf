"""Decode-step profiling driver: one captured decode graph of the serving engine.

    python -m kapsl_sdk_b200.utils.step_probe [--model qwen2.5-7b] [--batch 16] [--prompt 512]

Builds the engine on cuda:0 with random-init weights, prefills ``--batch``
requests of ``--prompt`` random tokens, runs a few decode steps, then replays
the decode graph of that batch: 3 warm-up and 20 timed replays (CUDA events),
printed as one JSON line.  One more replay runs inside the NVTX range
``probe_step``, the capture target for a per-kernel launch list:

    ncu --metrics gpu__time_duration.sum --clock-control none --nvtx --nvtx-include "probe_step/" \\
        --csv --log-file launches.csv python -m kapsl_sdk_b200.utils.step_probe
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="qwen2.5-7b")
    p.add_argument("--batch", type=int, default=16)
    p.add_argument("--prompt", type=int, default=512)
    a = p.parse_args()
    from .._ext import cuda_ops
    from ..llm.engine import EngineConfig, LLMEngine
    from ..llm.sequence import SamplingParams
    from ..models.config import get_preset

    cuda_ops()
    dev = torch.device("cuda", 0)
    cfg = get_preset(a.model)
    eng = LLMEngine(cfg, device=dev, engine_cfg=EngineConfig(
        max_num_seqs=max(64, a.batch), max_num_batched_tokens=max(2048, a.prompt), max_model_len=a.prompt + 512,
        num_blocks=a.batch * ((a.prompt + 512) // 16 + 1) + 64, overlap_steps=False), seed=0)
    rng = np.random.default_rng(0)
    for i in range(a.batch):
        eng.add_request(f"p{i}", rng.integers(0, cfg.vocab_size, a.prompt).tolist(),
                        SamplingParams(max_new_tokens=256, ignore_eos=True))
    r = eng.runner
    while True:  # prefill, until the next batch is a pure decode of every request
        batch = eng.scheduler.schedule()
        if not batch.prefill and len(batch.decode) == a.batch:
            break
        if batch.admitted:
            r.admit(batch.admitted)
        eng._complete(eng._launch(batch))
    eng._complete(eng._launch(batch))
    key = (r.graph_sizes[np.searchsorted(r.graph_sizes, a.batch)], False)
    g = r.graphs[key]
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(20):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    print(json.dumps({"model": a.model, "batch": a.batch, "graph_bucket": key[0], "kernel_nodes": r.graph_launches[key],
                      "ms_per_step": round(s.elapsed_time(e) / 20, 3)}), flush=True)
    torch.cuda.nvtx.range_push("probe_step")
    g.replay()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    eng.shutdown()


if __name__ == "__main__":
    main()
