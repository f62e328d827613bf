"""Device mesh, process groups and collective back-ends
(crates/kapsl-hal/src/device_mesh.rs, nccl_comm.rs, mock_comm.rs, distributed_ops.rs).

* ``MeshTopology``: data parallel, tensor parallel (degree, mesh shape),
  pipeline parallel (stages) or mixed (tp x pp x dp).
* ``DeviceMesh`` builds the named groups of the reference: ``tp_{i}``,
  ``pp_stage_{i}``, ``tp_dp{d}_pp{p}`` and ``world``.
* ``MeshComm`` implementations:
    - ``TorchComm``: ``torch.distributed`` over NCCL (GPU tensors, no host
      staging, one communicator per named group) or gloo (CPU);
    - ``MockComm``: ranks simulated in one process over shared state (tests);
      unlike the reference mock, all_reduce waits for every rank (bounded).
* ``DistributedOps``: typed helpers (all_reduce / all_gather / scatter / gather).
"""
from __future__ import annotations

import enum
import threading
import time
from dataclasses import dataclass, field
from typing import Optional

import numpy as np


class ReduceOp(enum.Enum):
    SUM = "sum"
    PROD = "prod"
    MIN = "min"
    MAX = "max"
    AVG = "avg"


@dataclass
class MeshTopology:
    kind: str = "data_parallel"   # data_parallel | tensor_parallel | pipeline_parallel | mixed
    tp: int = 1
    pp: int = 1
    dp: int = 1

    @classmethod
    def data_parallel(cls, n: int) -> "MeshTopology":
        return cls("data_parallel", 1, 1, n)

    @classmethod
    def tensor_parallel(cls, degree: int) -> "MeshTopology":
        return cls("tensor_parallel", degree, 1, 1)

    @classmethod
    def pipeline_parallel(cls, stages: int) -> "MeshTopology":
        return cls("pipeline_parallel", 1, stages, 1)

    @classmethod
    def mixed(cls, tp: int, pp: int, dp: int) -> "MeshTopology":
        return cls("mixed", tp, pp, dp)

    @property
    def world_size(self) -> int:
        return self.tp * self.pp * self.dp


@dataclass
class ProcessGroup:
    name: str
    ranks: list
    backend: str = "nccl"


class DeviceMesh:
    def __init__(self, topology: MeshTopology, rank: int = 0, comm=None):
        if not 0 <= rank < topology.world_size:
            raise ValueError(f"rank {rank} outside world of {topology.world_size}")
        self.topology = topology
        self.rank = rank
        self.comm = comm
        self.groups: dict = {"world": ProcessGroup("world", list(range(topology.world_size)))}
        t = topology
        # rank = ((d * pp) + p) * tp + t
        for d in range(t.dp):
            for p in range(t.pp):
                base = (d * t.pp + p) * t.tp
                ranks = list(range(base, base + t.tp))
                if t.kind in ("tensor_parallel", "mixed") and t.tp > 1:
                    name = f"tp_{d * t.pp + p}" if t.kind == "tensor_parallel" else f"tp_dp{d}_pp{p}"
                    self.groups[name] = ProcessGroup(name, ranks)
        if t.pp > 1:
            for p in range(t.pp):
                ranks = [(d * t.pp + p) * t.tp + x for d in range(t.dp) for x in range(t.tp)]
                self.groups[f"pp_stage_{p}"] = ProcessGroup(f"pp_stage_{p}", ranks)

    @property
    def world_size(self) -> int:
        return self.topology.world_size

    def coords(self, rank: Optional[int] = None) -> tuple:
        r = self.rank if rank is None else rank
        t = self.topology
        return (r // (t.pp * t.tp), (r // t.tp) % t.pp, r % t.tp)  # (dp, pp, tp)

    def group_of(self, prefix: str) -> Optional[ProcessGroup]:
        for g in self.groups.values():
            if g.name.startswith(prefix) and self.rank in g.ranks:
                return g
        return None


class MeshComm:
    """Collectives over numpy arrays (host) or torch tensors (device)."""

    rank: int
    world_size: int

    def all_reduce(self, x, op: ReduceOp = ReduceOp.SUM, group: str = "world"): ...
    def all_gather(self, x, group: str = "world"): ...
    def broadcast(self, x, root: int = 0, group: str = "world"): ...
    def reduce_scatter(self, x, op: ReduceOp = ReduceOp.SUM, group: str = "world"): ...
    def barrier(self, group: str = "world") -> None: ...
    def send(self, x, dst: int) -> None: ...
    def recv(self, like, src: int): ...


class TorchComm(MeshComm):
    """torch.distributed (nccl for CUDA tensors, gloo for CPU); one process group per named group."""

    def __init__(self, mesh: Optional[DeviceMesh] = None):
        import torch.distributed as dist

        self.dist = dist
        self.rank = dist.get_rank()
        self.world_size = dist.get_world_size()
        self._groups = {"world": None}
        if mesh is not None:
            for name, g in mesh.groups.items():
                if name != "world":
                    self._groups[name] = dist.new_group(g.ranks)

    def _g(self, group):
        return self._groups.get(group)

    def _op(self, op: ReduceOp):
        R = self.dist.ReduceOp
        return {ReduceOp.SUM: R.SUM, ReduceOp.PROD: R.PRODUCT, ReduceOp.MIN: R.MIN, ReduceOp.MAX: R.MAX,
                ReduceOp.AVG: R.SUM}[op]

    def all_reduce(self, x, op=ReduceOp.SUM, group="world"):
        self.dist.all_reduce(x, op=self._op(op), group=self._g(group))
        if op is ReduceOp.AVG:
            x /= self.dist.get_world_size(self._g(group))
        return x

    def all_gather(self, x, group="world"):
        import torch

        n = self.dist.get_world_size(self._g(group))
        out = [torch.empty_like(x) for _ in range(n)]
        self.dist.all_gather(out, x, group=self._g(group))
        return torch.cat(out)

    def broadcast(self, x, root=0, group="world"):
        self.dist.broadcast(x, src=root, group=self._g(group))
        return x

    def reduce_scatter(self, x, op=ReduceOp.SUM, group="world"):
        import torch

        n = self.dist.get_world_size(self._g(group))
        out = torch.empty(x.shape[0] // n, *x.shape[1:], dtype=x.dtype, device=x.device)
        self.dist.reduce_scatter_tensor(out, x, op=self._op(op), group=self._g(group))
        return out

    def barrier(self, group="world"):
        self.dist.barrier(group=self._g(group))

    def send(self, x, dst):
        self.dist.send(x, dst)

    def recv(self, like, src):
        self.dist.recv(like, src)
        return like


class _MockState:
    def __init__(self, world: int):
        self.world = world
        self.cv = threading.Condition()
        self.slots: dict = {}
        self.mailbox: dict = {}
        self.gen: dict = {}


class MockComm(MeshComm):
    """In-process simulated ranks (one thread per rank shares a state object)."""

    TIMEOUT_S = 10.0

    def __init__(self, rank: int, state: _MockState):
        self.rank = rank
        self.world_size = state.world
        self.s = state

    @staticmethod
    def create_group(world: int) -> list:
        st = _MockState(world)
        return [MockComm(r, st) for r in range(world)]

    def _exchange(self, key: str, value):
        s = self.s
        with s.cv:
            g = s.gen.get((key, self.rank), 0)
            s.gen[(key, self.rank)] = g + 1
            slot = s.slots.setdefault((key, g), {})
            slot[self.rank] = value
            s.cv.notify_all()
            deadline = time.monotonic() + self.TIMEOUT_S
            while len(slot) < s.world:
                left = deadline - time.monotonic()
                if left <= 0:
                    raise TimeoutError(f"rank {self.rank}: collective '{key}' timed out waiting for peers")
                s.cv.wait(left)
            vals = [slot[r] for r in range(s.world)]
            slot.setdefault("_done", set()).add(self.rank)
            if len(slot["_done"]) == s.world:
                del s.slots[(key, g)]
            return vals

    def all_reduce(self, x, op=ReduceOp.SUM, group="world"):
        vals = [np.asarray(v) for v in self._exchange("ar", np.array(x, copy=True))]
        f = {ReduceOp.SUM: np.sum, ReduceOp.PROD: np.prod, ReduceOp.MIN: np.min, ReduceOp.MAX: np.max,
             ReduceOp.AVG: np.mean}[op]
        return f(np.stack(vals), axis=0).astype(np.asarray(x).dtype)

    def all_gather(self, x, group="world"):
        return np.concatenate([np.asarray(v) for v in self._exchange("ag", np.array(x, copy=True))])

    def broadcast(self, x, root=0, group="world"):
        return np.asarray(self._exchange("bc", np.array(x, copy=True))[root])

    def reduce_scatter(self, x, op=ReduceOp.SUM, group="world"):
        full = self.all_reduce(x, op)
        n = full.shape[0] // self.world_size
        return full[self.rank * n:(self.rank + 1) * n]

    def barrier(self, group="world"):
        self._exchange("barrier", 0)

    def send(self, x, dst):
        with self.s.cv:
            self.s.mailbox.setdefault((self.rank, dst), []).append(np.array(x, copy=True))
            self.s.cv.notify_all()

    def recv(self, like, src):
        with self.s.cv:
            q = self.s.mailbox.setdefault((src, self.rank), [])
            deadline = time.monotonic() + self.TIMEOUT_S
            while not q:
                left = deadline - time.monotonic()
                if left <= 0:
                    raise TimeoutError(f"rank {self.rank}: recv from {src} timed out")
                self.s.cv.wait(left)
            return q.pop(0)


class DistributedOps:
    def __init__(self, comm: MeshComm):
        self.comm = comm

    def all_reduce_f32(self, x, op=ReduceOp.SUM):
        return self.comm.all_reduce(np.asarray(x, np.float32), op)

    def all_reduce_i32(self, x, op=ReduceOp.SUM):
        return self.comm.all_reduce(np.asarray(x, np.int32), op)

    def all_gather_f32(self, x):
        return self.comm.all_gather(np.asarray(x, np.float32))

    def scatter_f32(self, x, root: int = 0):
        """Root's buffer is split evenly; each rank gets its slice."""
        full = self.comm.broadcast(np.asarray(x, np.float32), root)
        n = full.shape[0] // self.comm.world_size
        return full[self.comm.rank * n:(self.comm.rank + 1) * n]

    def gather_f32(self, x):
        return self.comm.all_gather(np.asarray(x, np.float32))
