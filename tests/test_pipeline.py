"""Pipeline parallelism on CPU ranks (gloo): 2 and 3 stages with micro-batches
produce the same greedy tokens as one engine holding every layer."""
import json
import os
import socket
import subprocess
import sys
import textwrap

import pytest

from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
from kapsl_sdk_b200.llm.sequence import SamplingParams
from kapsl_sdk_b200.models.config import ModelConfig
from kapsl_sdk_b200.parallel.pp import split_batch, stage_layers

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def cfg():
    return ModelConfig(name="t", vocab_size=300, hidden_size=64, intermediate_size=128, num_layers=5, num_heads=4,
                       num_kv_heads=2, head_dim=16, max_position=512, bos_token_id=None, eos_token_id=None)


PROMPTS = [list(range(3, 3 + n)) for n in (40, 17, 64, 5, 33)]

WORKER = textwrap.dedent("""
    import json, os, sys
    sys.path.insert(0, {root!r})
    sys.path.insert(0, {tests!r})
    from datetime import timedelta
    import torch.distributed as dist
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.parallel.pp import PipelineStage
    from test_pipeline import cfg, PROMPTS
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    c = cfg()
    st = PipelineStage(rank, world, c.num_layers, micro_batches=2)
    eng = LLMEngine(c, device="cpu", engine_cfg=EngineConfig(max_num_seqs=8, max_num_batched_tokens=48,
                    max_model_len=256, num_blocks=128), seed=0, pp_stage=st)
    out = eng.generate(PROMPTS, SamplingParams.greedy(10, ignore_eos=True))
    print("OUT" + json.dumps({{"rank": rank, "layers": list(st.layers), "out": out}}), flush=True)
    dist.destroy_process_group()
""")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("stages", [2, 3])
def test_pipeline_matches_single_engine(stages):
    ref = LLMEngine(cfg(), device="cpu", engine_cfg=EngineConfig(max_num_seqs=8, max_num_batched_tokens=48,
                    max_model_len=256, num_blocks=128), seed=0).generate(PROMPTS,
                                                                           SamplingParams.greedy(10, ignore_eos=True))
    port = _port()
    script = WORKER.format(root=ROOT, tests=os.path.join(ROOT, "tests"))
    procs = [subprocess.Popen([sys.executable, "-c", script], stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                              text=True, env=dict(os.environ, RANK=str(r), WORLD_SIZE=str(stages),
                                                  MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port)))
             for r in range(stages)]
    res = []
    for p in procs:
        o, _ = p.communicate(timeout=240)
        assert p.returncode == 0, o[-3000:]
        res.append(json.loads([l for l in o.splitlines() if l.startswith("OUT")][0][3:]))
    layers = sum((r["layers"] for r in res), [])
    assert layers == list(range(5))
    for r in res:
        assert r["out"] == ref


def test_stage_split_and_microbatches():
    assert [list(stage_layers(10, 3, s)) for s in range(3)] == [[0, 1, 2, 3], [4, 5, 6], [7, 8, 9]]
    from kapsl_sdk_b200.llm.scheduler import ScheduledBatch

    class S:
        pass

    seqs = [S() for _ in range(5)]
    b = ScheduledBatch(decode=seqs[:3], prefill=[(seqs[3], 40), (seqs[4], 8)], admitted=[seqs[4]])
    parts = split_batch(b, 2)
    assert sum(len(p.decode) for p in parts) == 3 and sum(len(p.prefill) for p in parts) == 2
    assert [s for p in parts for s in p.admitted] == [seqs[4]]


WORKER_GPU = textwrap.dedent("""
    import json, os, sys
    sys.path.insert(0, {root!r})
    from datetime import timedelta
    import torch, torch.distributed as dist
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.config import ModelConfig
    from kapsl_sdk_b200.parallel.pp import PipelineStage
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    c = ModelConfig(name="s", arch="llama", vocab_size=2048, hidden_size=512, intermediate_size=1024, num_layers=5,
                    num_heads=4, num_kv_heads=2, head_dim=128, rope_theta=5e5, max_position=4096,
                    bos_token_id=None, eos_token_id=None)
    prompts = [list(range(5, 5 + n)) for n in (300, 77, 500, 16, 129)]
    ecfg = EngineConfig(max_num_seqs=8, max_num_batched_tokens=256, max_model_len=1024, num_blocks=300)
    st = PipelineStage(rank, world, c.num_layers, micro_batches=2)
    eng = LLMEngine(c, device=dev, engine_cfg=ecfg, seed=0, pp_stage=st)
    out = eng.generate(prompts, SamplingParams.greedy(12, ignore_eos=True))
    if rank == world - 1:
        ref = LLMEngine(c, device=dev, engine_cfg=EngineConfig(max_num_seqs=8, max_num_batched_tokens=256,
                        max_model_len=1024, num_blocks=300, use_cuda_graph=False), seed=0)
        want = ref.generate(prompts, SamplingParams.greedy(12, ignore_eos=True))
        agree = sum(int(a == b) for o, w in zip(out, want) for a, b in zip(o, w))
        print("AGREE", agree, sum(len(w) for w in want), flush=True)
        ref.shutdown()
    eng.shutdown()
    dist.destroy_process_group()
""")


@pytest.mark.gpu
def test_pipeline_two_gpus_matches_single_gpu():
    """Two pipeline stages on two GPUs (NCCL point-to-point hidden states,
    micro-batches) against one GPU holding every layer."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, "-c", WORKER_GPU.format(root=ROOT)], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            o, _ = p.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        outs.append((p.returncode, o))
    for rc, o in outs:
        assert rc == 0, o[-3000:]
    line = [l for l in outs[1][1].splitlines() if l.startswith("AGREE")][0]
    agree, total = (int(x) for x in line.split()[1:])
    assert agree >= 0.9 * total, line
