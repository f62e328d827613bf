"""Request scheduling in front of engines (L5).

* ``determine_priority`` — latency-critical vs throughput classification
  (crates/kapsl-scheduler/src/request_metadata.rs:5-102): explicit priority 0,
  SLA < 250 ms, light work (input <= 500 KB, <= 1 GFLOP, or size x batch <= 2 MB)
  or batch <= 4 are latency critical.
* ``WorkQueue`` / ``Executor`` — a bounded native queue per worker; high-priority
  requests run one at a time, low-priority ones are micro-batched up to
  ``max_micro_batch`` within ``queue_delay`` and sent to ``engine.infer_batch``
  (gpu_executor.rs:11-329).  Cancellation is checked before execution.
* ``Scheduler`` — ``num_devices x workers_per_device`` high/low queue pairs,
  a thread pool for ``force_cpu`` requests, overflow policy Block /
  DropNewest / DropOldest, ``try_infer`` never blocks, queue depth counts
  in-flight work, healthy while every queue is below 80% (scheduler.rs:14-410).
  ``infer_stream`` calls the engine directly (as the reference does).
"""
from __future__ import annotations

import concurrent.futures as cf
import enum
import threading
import time
from dataclasses import dataclass
from typing import Optional

from ..engine_api import EngineError, EngineMetrics, InferenceRequest
from .router import MeshRouter

LIGHT_TASK_SIZE_BYTES = 500_000
LIGHT_TASK_FLOPS = 1_000_000_000
COMBINED_WORK_THRESHOLD = 2_000_000
SLA_LATENCY_CRITICAL_MS = 250
SMALL_BATCH_SIZE = 4


class Priority(enum.Enum):
    LATENCY_CRITICAL = "latency"
    THROUGHPUT = "throughput"


@dataclass
class SchedMetadata:
    priority: int = 1
    sla_deadline_ms: Optional[int] = None
    batch_size: int = 1
    input_size_bytes: Optional[int] = None
    estimated_flops: Optional[int] = None


def determine_priority(m: SchedMetadata) -> Priority:
    if m.priority == 0:
        return Priority.LATENCY_CRITICAL
    if m.sla_deadline_ms is not None and m.sla_deadline_ms < SLA_LATENCY_CRITICAL_MS:
        return Priority.LATENCY_CRITICAL
    if m.input_size_bytes is not None and m.input_size_bytes <= LIGHT_TASK_SIZE_BYTES:
        return Priority.LATENCY_CRITICAL
    if m.estimated_flops is not None and m.estimated_flops <= LIGHT_TASK_FLOPS:
        return Priority.LATENCY_CRITICAL
    if m.input_size_bytes is not None and m.input_size_bytes * m.batch_size <= COMBINED_WORK_THRESHOLD:
        return Priority.LATENCY_CRITICAL
    if m.batch_size <= SMALL_BATCH_SIZE:
        return Priority.LATENCY_CRITICAL
    return Priority.THROUGHPUT


class OverflowPolicy(enum.Enum):
    BLOCK = "block"
    DROP_NEWEST = "drop_newest"
    DROP_OLDEST = "drop_oldest"


class _Job:
    __slots__ = ("request", "future", "enqueued")

    def __init__(self, request: InferenceRequest):
        self.request = request
        self.future: cf.Future = cf.Future()
        self.enqueued = time.perf_counter()


class WorkQueue:
    """Bounded queue of one executor worker.  The queueing itself (overflow policy,
    micro-batch take, depth, close) is the native ``WorkQueue``
    (csrc/native/work_queue.h), which waits with the GIL released; this wrapper
    fails the futures of jobs the DROP_OLDEST policy evicts."""

    _POLICY = {OverflowPolicy.BLOCK: 0, OverflowPolicy.DROP_NEWEST: 1, OverflowPolicy.DROP_OLDEST: 2}

    def __init__(self, capacity: int):
        from .._ext import native

        self.capacity = capacity
        self._q = native().WorkQueue(capacity)

    @property
    def closed(self) -> bool:
        return self._q.closed

    def depth(self) -> int:
        return self._q.depth()

    def put(self, job: _Job, policy: OverflowPolicy, block: bool = True) -> bool:
        ok, evicted = self._q.put(job, self._POLICY[policy], block)
        if evicted is not None:
            evicted.future.set_exception(EngineError.overloaded("request dropped: queue overflow"))
        return ok

    def take(self, max_items: int, delay_s: float) -> list:
        return self._q.take(max_items, delay_s)

    def done(self, n: int) -> None:
        self._q.done(n)

    def close(self) -> None:
        self._q.close()  # the executor still runs what is queued, then stops


class Executor:
    """Worker for one queue: high priority -> single requests, low -> micro-batches."""

    def __init__(self, engine, queue: WorkQueue, max_micro_batch: int, queue_delay_s: float, batched: bool):
        self.engine = engine
        self.queue = queue
        self.max_micro_batch = max_micro_batch if batched else 1
        self.delay = queue_delay_s if batched else 0.0
        self.thread = threading.Thread(target=self._run, daemon=True, name="kapsl-executor")
        self.batches = 0
        self.thread.start()

    def _run(self) -> None:
        while True:
            batch = self.queue.take(self.max_micro_batch, self.delay)
            if not batch:
                if self.queue.closed:
                    return
                continue
            live = []
            for j in batch:
                tok = j.request.cancellation
                if tok is not None and tok.is_cancelled():
                    j.future.set_exception(EngineError.cancelled("Request cancelled before execution"))
                else:
                    live.append(j)
            try:
                if len(live) == 1:
                    live[0].future.set_result(self.engine.infer(live[0].request))
                elif live:
                    outs = self.engine.infer_batch([j.request for j in live])
                    for j, o in zip(live, outs):
                        j.future.set_result(o)
                self.batches += 1
            except Exception as e:
                err = e if isinstance(e, EngineError) else EngineError.inference(str(e))
                for j in live:
                    if not j.future.done():
                        j.future.set_exception(err)
            finally:
                self.queue.done(len(batch))


class Scheduler:
    def __init__(self, engines: list, cpu_workers: int = 2, workers_per_device: int = 1, queue_size: int = 64,
                 overflow: OverflowPolicy = OverflowPolicy.BLOCK, max_micro_batch: int = 8,
                 queue_delay_ms: float = 2.0, mesh: Optional[MeshRouter] = None, cpu_engine=None):
        if not engines:
            raise ValueError("at least one engine is required")
        self.engines = engines
        self.overflow = overflow
        self.queue_size = queue_size
        self.router = mesh or MeshRouter.round_robin(len(engines) * workers_per_device)
        self.high: list = []
        self.low: list = []
        self.executors: list = []
        for dev, eng in enumerate(engines):
            for _ in range(workers_per_device):
                hq, lq = WorkQueue(queue_size), WorkQueue(queue_size)
                self.high.append(hq)
                self.low.append(lq)
                self.executors.append(Executor(eng, hq, 1, 0.0, batched=False))
                self.executors.append(Executor(eng, lq, max_micro_batch, queue_delay_ms / 1000.0, batched=True))
        self.cpu_engine = cpu_engine or engines[0]
        self.cpu_pool = cf.ThreadPoolExecutor(max_workers=max(1, cpu_workers), thread_name_prefix="kapsl-cpu")

    def _route(self, request: InferenceRequest) -> int:
        return self.router.route(request.session_id) % len(self.high)

    def _submit(self, request: InferenceRequest, priority: Priority, block: bool) -> cf.Future:
        if request.metadata is not None and request.metadata.force_cpu:
            return self.cpu_pool.submit(self.cpu_engine.infer, request)
        w = self._route(request)
        q = self.high[w] if priority is Priority.LATENCY_CRITICAL else self.low[w]
        job = _Job(request)
        if not q.put(job, self.overflow, block=block):
            raise EngineError.overloaded("queue full")
        return job.future

    def infer(self, request: InferenceRequest, priority: Priority = Priority.THROUGHPUT):
        if isinstance(priority, str):
            priority = Priority.LATENCY_CRITICAL if priority.startswith("lat") else Priority.THROUGHPUT
        fut = self._submit(request, priority, block=True)
        timeout = None
        if request.metadata is not None and request.metadata.timeout_ms:
            timeout = request.metadata.timeout_ms / 1000.0
        try:
            return fut.result(timeout=timeout)
        except cf.TimeoutError:
            raise EngineError.timeout(f"request exceeded {request.metadata.timeout_ms} ms")

    def try_infer(self, request: InferenceRequest, priority: Priority = Priority.THROUGHPUT) -> cf.Future:
        """Never blocks: raises Overloaded when the target queue is full."""
        return self._submit(request, priority, block=False)

    def infer_stream(self, request: InferenceRequest):
        if not self.is_healthy():
            raise EngineError.overloaded("scheduler unhealthy")
        eng = self.engines[self._route(request) % len(self.engines)]
        return eng.infer_stream(request)

    def infer_stream_native(self, request: InferenceRequest):
        """:meth:`infer_stream` as a native token channel when the routed engine
        offers one (token-id requests to an LLM backend), else None."""
        if not self.is_healthy():
            raise EngineError.overloaded("scheduler unhealthy")
        eng = self.engines[self._route(request) % len(self.engines)]
        native = getattr(eng, "infer_stream_native", None)
        return native(request) if native is not None else None

    def get_queue_depth(self) -> tuple:
        return sum(q.depth() for q in self.high), sum(q.depth() for q in self.low)

    def is_healthy(self) -> bool:
        """Every queue below 80% of its capacity (reference scheduler.rs:284-304),
        and no engine reporting itself unhealthy (e.g. a device fault)."""
        lim = 0.8 * self.queue_size
        if not all(q.depth() < lim for q in self.high + self.low):
            return False
        for e in self.engines:
            hc = getattr(e, "health_check", None)
            if hc is not None and not hc():
                return False
        return True

    def get_metrics(self) -> EngineMetrics:
        m = self.engines[0].metrics()
        h, l = self.get_queue_depth()
        m.queue_depth = h + l
        return m

    def shutdown(self) -> None:
        for q in self.high + self.low:
            q.close()
        self.cpu_pool.shutdown(wait=False)
