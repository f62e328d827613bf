"""Multi-GPU serving through the wire API: the launcher under torchrun with 2
ranks (tensor parallel over 2 GPUs; rank 0 serves a Unix socket and the other
rank follows its steps), streamed with KapslClient.infer_stream.  The served
greedy tokens equal the same TP2 engine driven directly (the serving path
adds nothing) and agree with one GPU (TP1) up to bf16 near-ties."""
import os
import signal
import socket
import subprocess
import sys
import threading
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_group_serves_over_socket(tmp_path):
    from kapsl_sdk import KapslClient
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.config import get_preset

    sock, ready = str(tmp_path / "kapsl.sock"), str(tmp_path / "ready")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_port()), "-m", "kapsl_sdk_b200.runtime.launch", "--preset",
           "tiny-qwen2", "--tp", "2", "--socket", sock, "--greedy", "--ignore-eos", "--max-new-tokens", "12",
           "--max-num-seqs", "8", "--max-batched-tokens", "256", "--max-model-len", "1024", "--ready-file", ready]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    proc = subprocess.Popen(cmd, cwd=ROOT, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                            start_new_session=True)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 4096, int(n)).tolist() for n in (40, 300, 7, 129)]
    got = [None] * len(prompts)
    try:
        t0 = time.time()
        while not os.path.exists(ready):
            assert proc.poll() is None, proc.communicate()[0][-4000:]
            assert time.time() - t0 < 300, "launcher did not come up"
            time.sleep(0.2)

        def run(i):
            c = KapslClient(sock)
            data = np.asarray(prompts[i], dtype=np.int32).tobytes()
            got[i] = [int(np.frombuffer(p, dtype=np.int32)[0])
                      for p in c.infer_stream(0, [1, len(prompts[i])], "int32", data)]

        th = [threading.Thread(target=run, args=(i,)) for i in range(len(prompts))]
        [t.start() for t in th]
        [t.join(180) for t in th]
    finally:
        # stop rank 0 only: it stops its followers, both exit 0 and so does torchrun (a
        # SIGTERM to torchrun itself makes its agent exit 1 however the workers end)
        try:
            leader = int(open(ready).read().split("\n")[2])
            os.kill(leader, signal.SIGTERM)
            out = proc.communicate(timeout=120)[0]
        except Exception:
            os.killpg(proc.pid, signal.SIGTERM)
            out = proc.communicate(timeout=120)[0]
    assert proc.returncode == 0, out[-4000:]
    assert all(g is not None and len(g) == 12 for g in got), (got, out[-3000:])
    d0 = [l for l in out.splitlines() if "rank 0: outputs" in l]
    d1 = [l for l in out.splitlines() if "rank 1: followed" in l]
    assert d0 and d1 and d0[0].split("outputs ")[1] == d1[0].split("outputs ")[1], out[-3000:]
    # one GPU (TP1) on the same random weights
    eng = LLMEngine(get_preset("tiny-qwen2"), device=torch.device("cuda", 0), engine_cfg=EngineConfig(
        max_num_seqs=8, max_num_batched_tokens=256, max_model_len=1024, num_blocks=512), seed=0)
    want = eng.generate(prompts, SamplingParams.greedy(12, ignore_eos=True))
    eng.shutdown()
    same = sum(a == b for x, y in zip(got, want) for a, b in zip(x, y))
    assert [g[0] for g in got] == [w[0] for w in want], (got, want)
    assert same >= 0.9 * sum(len(w) for w in want), (got, want)
