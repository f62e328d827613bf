"""CronScheduler: periodic inference jobs declared in a package manifest
(crates/kapsl-scheduler/src/cron_scheduler.rs:28-405, schema in
crates/kapsl-core/src/loader.rs:14-66).

A job fires on a fixed interval (``{"interval_secs": N}``) or a 6-field cron
expression ``<sec> <min> <hour> <dom> <mon> <dow>`` (``*``, lists, ranges and
``*/step``).  ``skip_if_busy`` uses the scheduler's non-blocking ``try_infer``
and counts a miss when the queue is full; ``block`` waits.  Counters and an
optional callback per firing.
"""
from __future__ import annotations

import datetime as _dt
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Optional

from ..engine_api import BinaryTensorPacket, EngineError, InferenceRequest, NamedTensor, RequestMetadata


def _parse_field(spec: str, lo: int, hi: int) -> set:
    out = set()
    for part in spec.split(","):
        step = 1
        if "/" in part:
            part, s = part.split("/", 1)
            step = int(s)
        if part in ("*", ""):
            a, b = lo, hi
        elif "-" in part:
            a, b = (int(x) for x in part.split("-", 1))
        else:
            a = b = int(part)
        if a < lo or b > hi or a > b or step < 1:
            raise ValueError(f"cron field '{spec}' out of range [{lo}, {hi}]")
        out.update(range(a, b + 1, step))
    return out


class CronExpression:
    def __init__(self, expr: str):
        f = expr.split()
        if len(f) != 6:
            raise ValueError("cron expression needs 6 fields: sec min hour dom mon dow")
        self.sec = _parse_field(f[0], 0, 59)
        self.min = _parse_field(f[1], 0, 59)
        self.hour = _parse_field(f[2], 0, 23)
        self.dom = _parse_field(f[3], 1, 31)
        self.mon = _parse_field(f[4], 1, 12)
        self.dow = _parse_field(f[5].replace("7", "0"), 0, 6)

    def matches(self, t: _dt.datetime) -> bool:
        return (t.second in self.sec and t.minute in self.min and t.hour in self.hour and t.day in self.dom
                and t.month in self.mon and (t.isoweekday() % 7) in self.dow)

    def next_after(self, t: _dt.datetime) -> _dt.datetime:
        c = t.replace(microsecond=0) + _dt.timedelta(seconds=1)
        for _ in range(366 * 24 * 3600):
            if self.matches(c):
                return c
            c += _dt.timedelta(seconds=1)
        raise ValueError("cron expression never fires")


@dataclass
class CronJob:
    id: str
    input: BinaryTensorPacket
    interval_s: Optional[float] = None
    expression: Optional[str] = None
    additional_inputs: list = field(default_factory=list)
    priority: str = "throughput"
    force_cpu: bool = False
    overflow: str = "skip_if_busy"
    fired: int = 0
    missed: int = 0
    errors: int = 0
    callback: Optional[Callable] = None

    def next_fire(self, now: float) -> float:
        if self.interval_s is not None:
            return now + self.interval_s
        t = _dt.datetime.fromtimestamp(now)
        return CronExpression(self.expression).next_after(t).timestamp()


class CronScheduler:
    def __init__(self, scheduler, clock=time.time):
        self.scheduler = scheduler
        self.clock = clock
        self.jobs: dict = {}
        self._next: dict = {}
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._lock = threading.Lock()

    def register(self, job: CronJob) -> None:
        if job.interval_s is None and job.expression is None:
            raise ValueError("cron job needs interval_secs or a cron expression")
        if job.expression is not None:
            CronExpression(job.expression)
        if job.interval_s is not None and job.interval_s <= 0:
            raise ValueError("interval_secs must be > 0")
        with self._lock:
            self.jobs[job.id] = job
            self._next[job.id] = job.next_fire(self.clock())

    def unregister(self, job_id: str) -> bool:
        with self._lock:
            self._next.pop(job_id, None)
            return self.jobs.pop(job_id, None) is not None

    def register_from_manifest(self, defs: list) -> int:
        from ..engine_api import TensorDtype

        n = 0
        for d in defs or []:
            sch = d.get("schedule")
            inp = d["input"]
            pkt = BinaryTensorPacket(list(inp["shape"]), TensorDtype.parse(inp["dtype"]), bytes(inp.get("data", b"")))
            job = CronJob(id=d["id"], input=pkt,
                          interval_s=float(sch["interval_secs"]) if isinstance(sch, dict) else None,
                          expression=sch if isinstance(sch, str) else None,
                          priority=d.get("priority", "throughput"), force_cpu=bool(d.get("force_cpu", False)),
                          overflow=d.get("overflow_policy", "skip_if_busy"))
            self.register(job)
            n += 1
        return n

    def list(self) -> list:
        return [{"id": j.id, "fired": j.fired, "missed": j.missed, "errors": j.errors} for j in self.jobs.values()]

    def fire(self, job: CronJob) -> None:
        req = InferenceRequest(job.input, [NamedTensor(n, t) for n, t in job.additional_inputs],
                               metadata=RequestMetadata(force_cpu=job.force_cpu))
        prio = "latency" if job.priority == "latency_critical" else "throughput"
        try:
            if job.overflow == "skip_if_busy":
                from .scheduler import Priority

                fut = self.scheduler.try_infer(req, Priority.LATENCY_CRITICAL if prio == "latency"
                                               else Priority.THROUGHPUT)
                out = fut.result()
            else:
                out = self.scheduler.infer(req, prio)
            job.fired += 1
            if job.callback:
                job.callback(job.id, out)
        except EngineError as e:
            if e.is_overloaded:
                job.missed += 1
            else:
                job.errors += 1

    def tick(self) -> int:
        """Fire every due job once; returns how many fired or were attempted."""
        now = self.clock()
        due = []
        with self._lock:
            for jid, t in self._next.items():
                if t <= now:
                    due.append(self.jobs[jid])
                    self._next[jid] = self.jobs[jid].next_fire(now)
        for j in due:
            self.fire(j)
        return len(due)

    def start(self, period_s: float = 0.05) -> None:
        def run():
            while not self._stop.wait(period_s):
                self.tick()

        self._stop.clear()
        self._thread = threading.Thread(target=run, daemon=True, name="kapsl-cron")
        self._thread.start()

    def stop(self) -> None:
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=5)
