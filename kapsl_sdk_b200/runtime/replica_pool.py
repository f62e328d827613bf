"""ReplicaPool: spreads requests over replicas of one model with failover
(crates/kapsl-scheduler/src/replica_pool.rs:8-557).

Strategies: RoundRobin, LeastLoaded, Sticky (session hash).  LeastLoaded is
KV-pressure aware when any healthy replica reports paged-KV metrics: replicas
are ordered by (pressure tier of block utilization: <70% / <85% / <95% / more,
queue depth, most free blocks, most free bytes, fewest requests); replicas
without KV metrics sort last.  On an error the request is retried on the other
healthy replicas in routing-key order (unary and streaming).

A replica is any object with ``infer(request, priority)``,
``infer_stream(request)``, ``get_queue_depth() -> (high, low)``,
``is_healthy()`` and ``get_metrics() -> EngineMetrics`` (a ``Scheduler``).
"""
from __future__ import annotations

import enum
import itertools
import threading
import zlib
from dataclasses import dataclass

from ..engine_api import EngineError, InferenceRequest


class PoolStrategy(enum.Enum):
    ROUND_ROBIN = "round_robin"
    LEAST_LOADED = "least_loaded"
    STICKY = "sticky"


@dataclass
class ReplicaStats:
    replica_id: int
    requests_total: int
    queue_depth: tuple
    healthy: bool


class _Replica:
    def __init__(self, rid: int, sched):
        self.replica_id = rid
        self.scheduler = sched
        self.requests_total = 0


def kv_routing_key(m):
    total = m.kv_cache_blocks_total
    if not total:
        return None
    free = min(m.kv_cache_blocks_free, total)
    permille = (total - free) * 1000 // max(total, 1)
    tier = 0 if permille < 700 else 1 if permille < 850 else 2 if permille < 950 else 3
    return tier, free, max(0, m.kv_cache_bytes_capacity - m.kv_cache_bytes_used)


class ReplicaPool:
    def __init__(self, strategy: PoolStrategy = PoolStrategy.ROUND_ROBIN):
        self.strategy = strategy
        self.replicas: list = []
        self._rr = itertools.count()
        self._lock = threading.RLock()

    # ------------------------------------------------------------- membership
    def add_replica(self, replica_id: int, scheduler) -> None:
        with self._lock:
            self.replicas.append(_Replica(replica_id, scheduler))

    def remove_replica(self, replica_id: int) -> bool:
        with self._lock:
            for i, r in enumerate(self.replicas):
                if r.replica_id == replica_id:
                    del self.replicas[i]
                    return True
        return False

    def size(self) -> int:
        return len(self.replicas)

    def healthy_count(self) -> int:
        return sum(1 for r in self.replicas if r.scheduler.is_healthy())

    def stats(self) -> list:
        return [ReplicaStats(r.replica_id, r.requests_total, r.scheduler.get_queue_depth(),
                             r.scheduler.is_healthy()) for r in self.replicas]

    # -------------------------------------------------------------- routing
    def _key(self, r: _Replica, memory_aware: bool):
        h, l = r.scheduler.get_queue_depth()
        depth = h + l
        if memory_aware:
            k = kv_routing_key(r.scheduler.get_metrics())
            if k is not None:
                tier, free_blocks, free_bytes = k
                return (tier, depth, -free_blocks, -free_bytes, r.requests_total)
            return (255, depth, 0, 0, r.requests_total)
        return (0, depth, 0, 0, r.requests_total)

    def _memory_aware(self, reps) -> bool:
        return any(kv_routing_key(r.scheduler.get_metrics()) is not None for r in reps if r.scheduler.is_healthy())

    def _ordered(self, request: InferenceRequest) -> list:
        with self._lock:
            reps = list(self.replicas)
        if not reps:
            raise EngineError.model_not_loaded()
        healthy = [r for r in reps if r.scheduler.is_healthy()] or reps
        if self.strategy is PoolStrategy.STICKY and request.session_id:
            first = reps[zlib.crc32(request.session_id.encode()) % len(reps)]
        elif self.strategy is PoolStrategy.LEAST_LOADED:
            ma = self._memory_aware(healthy)
            first = min(healthy, key=lambda r: self._key(r, ma))
        else:
            first = reps[next(self._rr) % len(reps)]
        ma = self._memory_aware(healthy)
        rest = sorted((r for r in healthy if r is not first), key=lambda r: self._key(r, ma))
        return [first] + rest

    # ------------------------------------------------------------- execution
    def infer(self, request: InferenceRequest, priority="throughput"):
        order = self._ordered(request)
        last = None
        for r in order:
            r.requests_total += 1
            try:
                return r.scheduler.infer(request, priority)
            except EngineError as e:
                if e.kind.name in ("INVALID_INPUT", "CANCELLED"):
                    raise  # not a replica failure
                last = e
        raise last

    execute = infer

    def infer_stream(self, request: InferenceRequest):
        return self._stream(request, native=False)

    def infer_stream_native(self, request: InferenceRequest):
        """:meth:`infer_stream` as a native token channel when the chosen replica
        offers one, else None; same ordering and failover."""
        return self._stream(request, native=True)

    def _stream(self, request: InferenceRequest, native: bool):
        order = self._ordered(request)
        last = None
        for r in order:
            if native and getattr(r.scheduler, "infer_stream_native", None) is None:
                return None
            r.requests_total += 1
            try:
                if native:
                    ch = r.scheduler.infer_stream_native(request)
                    if ch is None:
                        r.requests_total -= 1  # not applicable: the packet stream serves it
                    return ch
                return r.scheduler.infer_stream(request)
            except EngineError as e:
                if e.kind.name in ("INVALID_INPUT", "CANCELLED"):
                    raise
                last = e
        raise last

    def get_queue_depth(self) -> tuple:
        h = l = 0
        for r in self.replicas:
            a, b = r.scheduler.get_queue_depth()
            h, l = h + a, l + b
        return h, l

    def is_healthy(self) -> bool:
        return self.healthy_count() > 0
