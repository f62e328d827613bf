"""Multi-process serving (one process per rank): the launcher's rank 0 serves
KapslClient.infer_stream over a Unix socket and publishes every step's events
through the shared-memory step channel; the follower applies them and steps
in lock step.  On CPU ranks (gloo) each rank holds the whole model, so the
test checks the protocol: streamed tokens equal a single engine's, and every
rank ends with the same outputs."""
import os
import signal
import socket
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_step_channel_ring_and_backpressure():
    from kapsl_sdk_b200.parallel.group import StepChannel

    name = f"kapsl-test-{os.getpid()}"
    lead = StepChannel(name, 3, 0, slots=2, slot_bytes=64, timeout_s=0.5)
    f1, f2 = StepChannel(name, 3, 1), StepChannel(name, 3, 2)
    try:
        assert lead.publish(b"a") == 1 and lead.publish(b"bb") == 2
        with pytest.raises(TimeoutError):  # both slots hold unread messages
            lead.publish(b"c", timeout_s=0.05)
        assert f1.receive() == b"a" and f2.receive() == b"a"
        assert lead.publish(b"c") == 3
        assert [f1.receive(), f1.receive()] == [b"bb", b"c"]
        assert [f2.receive(), f2.receive()] == [b"bb", b"c"]
        with pytest.raises(TimeoutError):
            f1.receive(timeout_s=0.05)
        with pytest.raises(ValueError):
            lead.publish(b"x" * 65)
    finally:
        for c in (f1, f2, lead):
            c.close()


def test_two_rank_group_serves_over_socket(tmp_path):
    from kapsl_sdk import KapslClient
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.config import get_preset

    sock = str(tmp_path / "kapsl.sock")
    ready = str(tmp_path / "ready")
    port = _port()
    args = [sys.executable, "-m", "kapsl_sdk_b200.runtime.launch", "--preset", "tiny-llama", "--socket", sock,
            "--greedy", "--ignore-eos", "--max-new-tokens", "6", "--max-num-seqs", "4", "--max-batched-tokens",
            "64", "--max-model-len", "256", "--ready-file", ready, "--tp", "2"]
    env = dict(os.environ, WORLD_SIZE="2", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="",
               PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    procs = [subprocess.Popen(args, cwd=ROOT, env=dict(env, RANK=str(r), LOCAL_RANK=str(r)), stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True) for r in range(2)]
    try:
        t0 = time.time()
        while not os.path.exists(ready):
            assert all(p.poll() is None for p in procs), [p.communicate()[0][-3000:] for p in procs]
            assert time.time() - t0 < 240, "launcher did not come up"
            time.sleep(0.2)
        rng = np.random.default_rng(3)
        prompts = [rng.integers(3, 32000, int(n)).tolist() for n in (40, 7, 90)]
        got = [None] * len(prompts)

        def run(i):
            c = KapslClient(sock)
            data = np.asarray(prompts[i], dtype=np.int32).tobytes()
            got[i] = [int(np.frombuffer(p, dtype=np.int32)[0])
                      for p in c.infer_stream(0, [1, len(prompts[i])], "int32", data)]

        th = [threading.Thread(target=run, args=(i,)) for i in range(len(prompts))]
        [t.start() for t in th]
        [t.join(120) for t in th]
        procs[0].send_signal(signal.SIGTERM)
        outs = [p.communicate(timeout=120)[0] for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert [p.returncode for p in procs] == [0, 0], [o[-3000:] for o in outs]
    eng = LLMEngine(get_preset("tiny-llama"), device="cpu", engine_cfg=EngineConfig(
        max_num_seqs=4, max_num_batched_tokens=64, max_model_len=256), seed=0)
    want = eng.generate(prompts, SamplingParams.greedy(6, ignore_eos=True))
    assert got == want
    d0 = [l for l in outs[0].splitlines() if "rank 0: outputs" in l][0].split("outputs ")[1]
    d1 = [l for l in outs[1].splitlines() if "rank 1: followed" in l][0].split("outputs ")[1]
    assert d0 == d1 and d0.startswith("3:"), (d0, d1)
