"""Failure detection with faults injected on the host (no GPU involved): a rank
that dies, a rank that never joins a collective, corrupted and truncated
frames and dropped connections at the socket server, and KV admission limits."""
import os
import socket
import struct
import subprocess
import sys
import tempfile
import textwrap
import time

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


HB_WORKER = textwrap.dedent("""
    import os, sys, time
    sys.path.insert(0, {root!r})
    from datetime import timedelta
    import torch.distributed as dist
    from kapsl_sdk_b200.parallel.health import HeartbeatMonitor, RankFailure
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=timedelta(seconds=20))
    store = dist.distributed_c10d._get_default_store()
    hb = HeartbeatMonitor(store, rank, world, interval_s=0.2, timeout_s=3.0).start()
    dist.barrier()
    if rank == 2:
        os._exit(17)  # crash between steps, no cleanup
    t0 = time.time()
    while True:  # the serving loop: one "step" per 50 ms, health check between steps
        time.sleep(0.05)
        try:
            hb.check()
        except RankFailure as e:
            print("DETECTED", e.ranks, round(time.time() - t0, 2), flush=True)
            break
        if time.time() - t0 > 30:
            print("MISSED", flush=True)
            break
    hb.stop()
    os._exit(0)
""")


def _spawn(script: str, world: int, timeout: float = 60.0):
    port = _port()
    procs = [subprocess.Popen([sys.executable, "-c", script], stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                              text=True, env=dict(os.environ, RANK=str(r), WORLD_SIZE=str(world),
                                                  MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port)))
             for r in range(world)]
    outs = []
    for p in procs:
        try:
            o, _ = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        outs.append((p.returncode, o))
    return outs


def test_dead_rank_is_detected_between_steps():
    outs = _spawn(HB_WORKER.format(root=ROOT), 3)
    assert outs[2][0] == 17
    for rc, o in outs[:2]:
        assert rc == 0 and "DETECTED [2]" in o, o[-2000:]
        detect_s = float(o.split("DETECTED [2]")[1].split()[0])
        assert detect_s < 10


NOJOIN_WORKER = textwrap.dedent("""
    import os, sys, time
    from datetime import timedelta
    import torch, torch.distributed as dist
    rank = int(os.environ["RANK"])
    dist.init_process_group("gloo", timeout=timedelta(seconds=3))
    if rank == 1:
        time.sleep(20)  # never joins the collective in time
        os._exit(0)
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(4))
        print("NO_ERROR", flush=True)
    except Exception as e:
        print("RAISED", type(e).__name__, round(time.time() - t0, 1), flush=True)
    os._exit(0)
""")


def test_collective_with_missing_rank_raises_instead_of_hanging():
    outs = _spawn(NOJOIN_WORKER, 2)
    assert "RAISED" in outs[0][1], outs[0][1][-2000:]
    # the 3 s process-group timeout ends the collective long before the peer would exit
    assert float(outs[0][1].split("RAISED")[1].split()[1]) < 15


def test_server_survives_corrupted_truncated_and_dropped_requests():
    from kapsl_sdk import KapslClient
    from kapsl_sdk_b200.engine_api import BinaryTensorPacket, Engine, TensorDtype
    from kapsl_sdk_b200.server import KapslServer

    class Echo(Engine):
        def infer(self, request):
            return request.input

        def load(self, path):
            pass

        def unload(self):
            pass

    d = tempfile.mkdtemp(prefix="kapsl-fd-")
    path = os.path.join(d, "s.sock")
    srv = KapslServer(models={0: Echo()}).listen_unix(path).start()
    try:
        def raw(payload: bytes, header=None):
            s = socket.socket(socket.AF_UNIX)
            s.connect(path)
            s.sendall(header if header is not None else struct.pack("<III", 0, 1, len(payload)))
            s.sendall(payload)
            return s

        # 1) garbage payload -> ERR frame, connection still usable by the server
        s = raw(b"\xff" * 40)
        hdr = s.recv(8)
        status = struct.unpack("<II", hdr)[0] if len(hdr) == 8 else None
        s.close()
        assert status == 1
        # 2) header announces more bytes than sent, then the client disconnects
        s = raw(b"\x00" * 10, header=struct.pack("<III", 0, 1, 1000))
        s.close()
        # 3) connect and drop immediately
        s = socket.socket(socket.AF_UNIX)
        s.connect(path)
        s.close()
        time.sleep(0.2)
        # the server keeps serving well-formed requests
        c = KapslClient(path)
        out = c.infer(0, [1, 4], "float32", np.arange(4, dtype=np.float32).tobytes())
        assert np.frombuffer(out, np.float32).tolist() == [0, 1, 2, 3]
    finally:
        srv.stop()


def test_kv_admission_limits():
    from kapsl_sdk_b200.engine_api import EngineError
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.config import ModelConfig

    cfg = ModelConfig(name="t", vocab_size=300, hidden_size=64, intermediate_size=128, num_layers=2, num_heads=4,
                      num_kv_heads=2, head_dim=16, max_position=512)
    eng = LLMEngine(cfg, device="cpu", engine_cfg=EngineConfig(max_num_seqs=4, max_num_batched_tokens=32,
                    max_model_len=512, num_blocks=8), seed=0)  # 8 blocks x 16 tokens
    with pytest.raises(EngineError) as e:
        eng.add_request("big", list(range(3, 200)), SamplingParams(max_new_tokens=100), admission_control=True)
    assert "ResourceExhausted" in type(e.value).__name__ or "hard limit" in str(e.value)
    eng.add_request("a", list(range(3, 50)), SamplingParams(max_new_tokens=40), admission_control=True)
    with pytest.raises(EngineError, match="soft limit"):
        eng.add_request("b", list(range(3, 40)), SamplingParams(max_new_tokens=10), admission_control=True)


@pytest.mark.gpu
def test_peer_wait_runs_out_and_engine_reports_failure():
    """(1) The fused tensor-parallel reduction on one GPU with world 2, the 'peer'
    a second local allocation whose flags nothing posts, and a 1 ms wait limit:
    the kernel returns within milliseconds and records status 32/33 instead of
    hanging.  (2) An engine whose step reads back such a status raises an
    EngineError naming it and reports itself unhealthy from then on."""
    import torch

    from kapsl_sdk_b200 import ops
    from kapsl_sdk_b200._ext import cuda_ops
    from kapsl_sdk_b200.engine_api import EngineError
    from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
    from kapsl_sdk_b200.llm.sequence import SamplingParams
    from kapsl_sdk_b200.models.config import ModelConfig

    c = cuda_ops()
    dev = torch.device("cuda", 0)
    rows, cols, W = 64, 256, 2
    part = [torch.zeros(rows, cols, dtype=torch.bfloat16, device=dev) for _ in range(W)]
    hid = [torch.zeros(rows, cols, dtype=torch.bfloat16, device=dev) for _ in range(W)]
    flags = [torch.zeros(32, dtype=torch.int64, device=dev) for _ in range(W)]
    epoch = torch.zeros(16, dtype=torch.int64, device=dev)
    err = ops.error_buffer(dev)
    err.zero_()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    c.tp_pull_reduce_ag([p.data_ptr() for p in part], [h.data_ptr() for h in hid], [f.data_ptr() for f in flags],
                        0, rows // W, rows, cols, cols, epoch, err, 1_000_000)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 2.0
    code = int(err.max())
    assert code in (32, 33), code
    err.zero_()
    torch.cuda.synchronize()

    cfg = ModelConfig(name="small", arch="qwen2", vocab_size=2048, hidden_size=512, intermediate_size=1024,
                      num_layers=2, num_heads=4, num_kv_heads=2, head_dim=128, rope_theta=1e6, rms_eps=1e-6,
                      max_position=4096, bos_token_id=None, eos_token_id=None)
    eng = LLMEngine(cfg, device=dev, engine_cfg=EngineConfig(max_num_seqs=4, max_num_batched_tokens=128,
                                                             max_model_len=512, num_blocks=64), seed=0)
    eng.add_request("a", list(range(10, 50)), SamplingParams.greedy(32, ignore_eos=True))
    eng.step()
    assert eng.health_check()
    err.fill_(32)  # stands in for a peer wait that ran out during the next step
    with pytest.raises(EngineError, match="missed barrier 1"):
        for _ in range(3):
            eng.step()
    assert not eng.health_check()
    with pytest.raises(EngineError):
        eng.step()
    assert int(err.max()) == 0  # the status was consumed
    eng.failed = None
    eng.shutdown()


def test_init_distributed_configures_the_collective_watchdog(monkeypatch):
    """The serving group's process group gets the timeout, and NCCL groups the
    watchdog setting that aborts failed or timed-out communicators."""
    import torch.distributed as dist

    from kapsl_sdk_b200.parallel import health

    seen = {}
    monkeypatch.setattr(dist, "init_process_group", lambda backend, **kw: seen.update(backend=backend, **kw))
    monkeypatch.delenv("TORCH_NCCL_ASYNC_ERROR_HANDLING", raising=False)
    health.init_distributed("nccl", 7.5, device="cuda:0")
    assert seen["backend"] == "nccl" and seen["timeout"].total_seconds() == 7.5 and seen["device_id"] == "cuda:0"
    import os
    assert os.environ["TORCH_NCCL_ASYNC_ERROR_HANDLING"] == "1"
    seen.clear()
    health.init_distributed("gloo", 3.0, device="cpu")
    assert seen == {"backend": "gloo", "timeout": seen["timeout"]} and seen["timeout"].total_seconds() == 3.0
