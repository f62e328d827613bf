"""MeshRouter: which worker serves a request
(crates/kapsl-scheduler/src/mesh_routing.rs:12-208).

Round-robin by default; a ``session_id`` hashes to a sticky worker; under a
tensor-parallel mesh requests go to the first worker of a TP group (the group
acts as one engine); pipeline-parallel meshes always enter at stage 0.
"""
from __future__ import annotations

import itertools
import threading
import zlib
from typing import Optional


class MeshRouter:
    def __init__(self, num_workers: int, mode: str = "round_robin", tp_degree: int = 1):
        if num_workers < 1:
            raise ValueError("num_workers must be >= 1")
        self.n = num_workers
        self.mode = mode
        self.tp = max(1, tp_degree)
        self._rr = itertools.count()
        self._lock = threading.Lock()

    @classmethod
    def round_robin(cls, n: int) -> "MeshRouter":
        return cls(n, "round_robin")

    @classmethod
    def tensor_parallel(cls, n: int, degree: int) -> "MeshRouter":
        return cls(n, "tensor_parallel", degree)

    @classmethod
    def pipeline(cls, n: int) -> "MeshRouter":
        return cls(n, "pipeline")

    @staticmethod
    def session_hash(session_id: str) -> int:
        return zlib.crc32(session_id.encode())

    def route(self, session_id: Optional[str] = None) -> int:
        if self.mode == "pipeline":
            return 0
        groups = max(1, self.n // self.tp) if self.mode == "tensor_parallel" else self.n
        if session_id:
            g = self.session_hash(session_id) % groups
        else:
            with self._lock:
                g = next(self._rr) % groups
        return g * self.tp if self.mode == "tensor_parallel" else g
