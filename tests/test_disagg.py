"""Disaggregated prefill/decode: two ranks (prefill, decode) serve greedy
requests through the KV connector and must produce the same tokens as one
engine doing both phases.  CPU engines over gloo move the pages through the
control store ("host" mode); the GPU test runs the P2P push kernel and the
copy-engine baseline between two GPUs."""
import os
import socket
import subprocess
import sys
import textwrap

import pytest
import torch

from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
from kapsl_sdk_b200.llm.sequence import SamplingParams
from kapsl_sdk_b200.models.config import ModelConfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def tiny_cfg():
    return ModelConfig(name="t", arch="llama", vocab_size=300, hidden_size=64, intermediate_size=128, num_layers=2,
                       num_heads=4, num_kv_heads=2, head_dim=16, rope_theta=10000.0, max_position=512,
                       bos_token_id=None, eos_token_id=None)


PROMPTS = [list(range(3, 3 + n)) for n in (40, 17, 64, 5)]

WORKER_CPU = textwrap.dedent("""
    import os, sys, json
    sys.path.insert(0, {root!r})
    import torch, torch.distributed as dist
    from datetime import timedelta
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.parallel.disagg import serve_disaggregated
    sys.path.insert(0, {tests!r})
    from test_disagg import tiny_cfg, PROMPTS
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    def make(role, group, gi, n):
        return LLMEngine(tiny_cfg(), device="cpu", engine_cfg=EngineConfig(max_num_seqs=4, max_num_batched_tokens=32,
                         max_model_len=256, num_blocks=64), seed=0)
    eng, outs, seqs = serve_disaggregated(make, PROMPTS, SamplingParams.greedy(12, ignore_eos=True), mode="host",
                                          timeout_s=60)
    if outs is not None:
        print("OUT" + json.dumps(outs), flush=True)
    dist.destroy_process_group()
""")


def _launch(script: str, world: int, extra_env=None, timeout=180):
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port))
        env.update(extra_env or {})
        procs.append(subprocess.Popen([sys.executable, "-c", script], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            o, _ = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        outs.append((p.returncode, o))
    for rc, o in outs:
        assert rc == 0, o[-3000:]
    return [o for _, o in outs]


def _reference_outputs(device="cpu"):
    eng = LLMEngine(tiny_cfg(), device=device, engine_cfg=EngineConfig(max_num_seqs=4, max_num_batched_tokens=32,
                    max_model_len=256, num_blocks=64), seed=0)
    return eng.generate(PROMPTS, SamplingParams.greedy(12, ignore_eos=True))


@pytest.mark.parametrize("world", [2, 4])
def test_disaggregated_cpu_matches_single_engine(world):
    """world 4: two prefill and two decode ranks (replicated CPU engines stand in for
    tensor-parallel ranks), which exercises the group leaders, broadcasts and the
    all-ranks completion protocol."""
    import json

    script = WORKER_CPU.format(root=ROOT, tests=os.path.join(ROOT, "tests"))
    outs = _launch(script, world)
    ref = _reference_outputs()
    for r in range(world // 2, world):
        line = [l for l in outs[r].splitlines() if l.startswith("OUT")][0]
        assert json.loads(line[3:]) == ref


def test_block_runs():
    from kapsl_sdk_b200.parallel.disagg import _runs

    assert _runs([4, 5, 6, 9, 10, 2]) == [(0, 4, 3), (3, 9, 2), (5, 2, 1)]
    assert _runs([]) == []


WORKER_GPU = textwrap.dedent("""
    import os, sys, json
    sys.path.insert(0, {root!r})
    import torch, torch.distributed as dist
    from datetime import timedelta
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.config import ModelConfig
    from kapsl_sdk_b200.models.llama import random_weights
    from kapsl_sdk_b200.parallel.disagg import serve_disaggregated
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    cfg = ModelConfig(name="s", arch="llama", vocab_size=2048, hidden_size=512, intermediate_size=1024, num_layers=2,
                      num_heads=4, num_kv_heads=2, head_dim=128, rope_theta=5e5, max_position=4096,
                      bos_token_id=None, eos_token_id=None)
    prompts = [list(range(5, 5 + n)) for n in (300, 77, 1000, 16)]
    def make(role, group, gi, n):
        w = random_weights(cfg, dev, seed=0, std=0.05)
        return LLMEngine(cfg, weights=w, device=dev, engine_cfg=EngineConfig(max_num_seqs=8,
                         max_num_batched_tokens=256, max_model_len=2048, num_blocks=400,
                         shareable_kv=(role == "decode")))
    eng, outs, seqs = serve_disaggregated(make, prompts, SamplingParams.greedy(10, ignore_eos=True),
                                          mode=os.environ["PD_MODE"], timeout_s=120)
    if outs is not None:
        ref = LLMEngine(cfg, weights=random_weights(cfg, dev, seed=0, std=0.05), device=dev,
                        engine_cfg=EngineConfig(max_num_seqs=8, max_num_batched_tokens=256, max_model_len=2048,
                                                num_blocks=400)).generate(prompts, SamplingParams.greedy(10,
                                                                          ignore_eos=True))
        agree = sum(int(a == b) for o, r in zip(outs, ref) for a, b in zip(o, r))
        print("AGREE", agree, sum(len(r) for r in ref), flush=True)
    eng.shutdown()
    dist.destroy_process_group()
""")


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["p2p", "copy"])
def test_disaggregated_two_gpus(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = WORKER_GPU.format(root=ROOT)
    outs = _launch(script, 2, {"PD_MODE": mode, "NCCL_NVLS_ENABLE": "0"}, timeout=300)
    line = [l for l in outs[1].splitlines() if l.startswith("AGREE")][0]
    agree, total = (int(x) for x in line.split()[1:])
    assert agree >= 0.9 * total, line
