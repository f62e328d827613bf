"""``kapsl-runtime``-style launcher: serve LLM model packages over the Unix
socket, TCP and shared-memory transports, on one GPU or on a tensor-parallel
group of GPUs (one process per GPU).

    python -m kapsl_sdk_b200.runtime.launch model.aimod
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m kapsl_sdk_b200.runtime.launch --tp 8 model.aimod --socket /tmp/kapsl.sock
    python -m kapsl_sdk_b200.runtime.launch --preset qwen2.5-7b      (random-init weights)

Flags follow the reference runtime: ``--socket`` (default ``/tmp/kapsl.sock``),
``--tcp-port`` (9096 when given without a value; off by default), ``--shm-name``
(``kapsl-shm-default`` when given without a value), ``--api-token`` (clients
must send it; reference crates/kapsl-ipc/src/server.rs:122 and
crates/kapsl-pyo3/src/lib.rs:24,28).  Serving parallelism comes from the
launch: ``WORLD_SIZE`` ranks form one tensor-parallel (or, for MoE models,
expert-parallel) group; ``--tp`` must equal it.  Rank 0 serves; the other
ranks follow its steps (:mod:`kapsl_sdk_b200.parallel.group`).  Model ids are
positions on the command line (one model per group when ``--tp`` > 1).

Environment keys (also read when the flags are absent): ``KAPSL_TP``,
``KAPSL_TP_MODE`` (fused | nccl), ``KAPSL_API_TOKEN``.
"""
from __future__ import annotations

import argparse
import os
import signal
import sys
import time
from typing import Optional

from ..server import DEFAULT_SHM_NAME, DEFAULT_SOCKET, DEFAULT_TCP_PORT


def parse_args(argv: Optional[list] = None) -> argparse.Namespace:
    p = argparse.ArgumentParser(prog="kapsl-runtime", description=__doc__.split("\n\n")[0])
    p.add_argument("models", nargs="*", help="model packages (.aimod), model files or directories; id = position")
    p.add_argument("--preset", action="append", default=[],
                   help="serve random-init weights of a named architecture (benchmarks); repeatable")
    p.add_argument("--socket", default=DEFAULT_SOCKET, help="Unix socket path ('' disables)")
    p.add_argument("--tcp-port", type=int, nargs="?", const=DEFAULT_TCP_PORT, default=None)
    p.add_argument("--tcp-host", default="127.0.0.1")
    p.add_argument("--shm-name", nargs="?", const=DEFAULT_SHM_NAME, default=None)
    p.add_argument("--shm-size", type=int, default=256 << 20)
    p.add_argument("--api-token", default=os.environ.get("KAPSL_API_TOKEN"))
    p.add_argument("--tp", type=int, default=int(os.environ.get("KAPSL_TP", "0")),
                   help="tensor-parallel degree; must equal WORLD_SIZE (0 = WORLD_SIZE)")
    p.add_argument("--tp-mode", default=os.environ.get("KAPSL_TP_MODE", "fused"), choices=["fused", "nccl"])
    p.add_argument("--pg-timeout", type=float, default=float(os.environ.get("KAPSL_PG_TIMEOUT", "120")),
                   help="seconds after which a stuck collective of the serving group is aborted")
    p.add_argument("--max-num-seqs", type=int, default=0)
    p.add_argument("--max-batched-tokens", type=int, default=0)
    p.add_argument("--max-model-len", type=int, default=0)
    p.add_argument("--ignore-eos", action="store_true", help="default sampling ignores EOS (benchmarks)")
    p.add_argument("--greedy", action="store_true", help="default sampling is greedy (temperature 0)")
    p.add_argument("--max-new-tokens", type=int, default=0, help="default max_new_tokens of requests")
    p.add_argument("--ready-file", default=None,
                   help="written by rank 0 once the servers accept connections: socket, TCP port and its pid, "
                        "one per line (SIGTERM to that pid stops the whole group)")
    a = p.parse_args(argv)
    if not a.models and not a.preset:
        p.error("give at least one model package / path or --preset")
    return a


def output_digest(engine) -> str:
    """Hash of every finished sequence's (request id, output ids): equal on all
    ranks of a group that stepped in lock step."""
    import hashlib

    h = hashlib.sha1()
    for s in sorted(engine.finished, key=lambda q: q.request_id):
        h.update(s.request_id.encode())
        h.update(repr(s.output_ids).encode())
    return f"{len(engine.finished)}:{h.hexdigest()[:16]}"


def _build(a, spec: str, is_preset: bool, dev, tp_comm):
    """(engine, tokenizer, runtime config) for one model."""
    from ..llm.backend import RuntimeConfig
    from ..llm.engine import EngineConfig, LLMEngine
    from ..models.config import get_preset
    from .loader import build_llm_engine

    if is_preset:
        cfg = get_preset(spec)
        e = EngineConfig(max_num_seqs=a.max_num_seqs or 256, max_num_batched_tokens=a.max_batched_tokens or 2048,
                         max_model_len=a.max_model_len or min(cfg.max_position, 4096))
        eng = LLMEngine(cfg, device=dev, engine_cfg=e, tp_comm=tp_comm, seed=0)
        tok, rc = None, RuntimeConfig()
    else:
        if any((a.max_num_seqs, a.max_batched_tokens, a.max_model_len)):
            raise SystemExit("--max-num-seqs / --max-batched-tokens / --max-model-len apply to --preset; "
                             "packages take them from their manifest")
        eng, tok, rc = build_llm_engine(spec, device=str(dev), tp_comm=tp_comm)
    if a.ignore_eos:
        rc.sampling.ignore_eos = True
    if a.greedy:
        rc.sampling.temperature, rc.sampling.top_k, rc.sampling.top_p = 0.0, 0, 1.0
        rc.sampling.repetition_penalty = 1.0
    if a.max_new_tokens:
        rc.sampling.max_new_tokens = a.max_new_tokens
    return eng, tok, rc


def main(argv: Optional[list] = None) -> int:
    a = parse_args(argv)
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    tp = a.tp or world
    if tp != world:
        raise SystemExit(f"--tp {tp} but WORLD_SIZE {world}: launch one process per GPU of the group")
    specs = [(m, False) for m in a.models] + [(m, True) for m in a.preset]
    if world > 1 and len(specs) != 1:
        raise SystemExit("a tensor-parallel group serves one model")
    cuda = torch.cuda.is_available()
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(dev)
    tp_comm = None
    if world > 1:
        from ..parallel.health import init_distributed
        from ..parallel.tp import TPComm

        init_distributed("nccl" if cuda else "gloo", a.pg_timeout, dev if cuda else None)
        tp_comm = TPComm.from_world(mode=a.tp_mode) if cuda else None
    from .._ext import cuda_ops

    if cuda:
        cuda_ops()  # the kernels must load on a GPU box
    built = [_build(a, s, pre, dev, tp_comm) for s, pre in specs]
    rc_code = 0
    if world > 1:
        import torch.distributed as dist

        from ..parallel.group import GroupLeader, StepChannel, follow

        name = [f"kapsl-group-{os.getpid()}-{os.urandom(4).hex()}" if rank == 0 else None]
        dist.broadcast_object_list(name, src=0)
        if rank != 0:
            chan = StepChannel(name[0], world, rank)
            # a termination signal reaches every rank at once: keep following until the
            # leader publishes its stop, and give up only if it has not after 30 s
            term = []
            signal.signal(signal.SIGTERM, lambda *_: term.append(time.monotonic()))
            signal.signal(signal.SIGINT, lambda *_: term.append(time.monotonic()))
            dist.barrier()
            try:
                steps = follow(built[0][0], chan, should_exit=lambda: bool(term) and time.monotonic() - term[0] > 30)
                print(f"kapsl-runtime rank {rank}: followed {steps} steps, outputs {output_digest(built[0][0])}",
                      flush=True)
                built[0][0].shutdown()
            finally:
                chan.close()
                dist.barrier()
                dist.destroy_process_group()
            return 0
        chan = StepChannel(name[0], world, 0)
        dist.barrier()
        built[0] = (GroupLeader(built[0][0], chan),) + tuple(built[0][1:])
    from ..llm.backend import LLMBackend
    from ..server import KapslServer

    backends = {i: LLMBackend(eng, tokenizer=tok, runtime_config=rc, own_thread=i > 0)
                for i, (eng, tok, rc) in enumerate(built)}
    srv = KapslServer(backends, api_token=a.api_token)
    if a.socket:
        srv.listen_unix(a.socket)
    if a.tcp_port is not None:
        srv.listen_tcp(a.tcp_host, a.tcp_port)
    if a.shm_name:
        srv.serve_shm(a.shm_name, a.shm_size)
    srv.start()
    first = backends[0]

    def _stop(*_):
        first._stop.set()

    signal.signal(signal.SIGTERM, _stop)
    signal.signal(signal.SIGINT, _stop)
    if a.ready_file:
        with open(a.ready_file + ".tmp", "w") as f:
            f.write(f"{a.socket or ''}\n{srv.tcp_port or ''}\n{os.getpid()}\n")  # socket, TCP port, rank 0 pid
        os.replace(a.ready_file + ".tmp", a.ready_file)
    print(f"kapsl-runtime: serving {len(backends)} model(s) on "
          f"{', '.join(x for x in (a.socket, f'tcp {srv.tcp_port}' if srv.tcp_port else '', a.shm_name) if x)}"
          f"{f' (tp {world})' if world > 1 else ''}", flush=True)
    try:
        first.run()  # model 0's engine loop on this thread until SIGTERM / SIGINT
    finally:
        srv.stop()
        eng0 = built[0][0]
        digest = output_digest(getattr(eng0, "engine", eng0))
        for b in backends.values():
            b.unload()
        print(f"kapsl-runtime rank 0: outputs {digest}", flush=True)
        if world > 1:
            import torch.distributed as dist

            chan.close()
            dist.barrier()
            dist.destroy_process_group()
    return rc_code


if __name__ == "__main__":
    sys.exit(main())
