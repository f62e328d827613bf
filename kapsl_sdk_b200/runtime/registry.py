"""ModelRegistry: loaded models, replicas, status with validated transitions,
status history with rollback, listeners and per-model latency percentiles
(crates/kapsl-core/src/model_registry.rs:6-404)."""
from __future__ import annotations

import enum
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Optional


class ModelStatus(enum.Enum):
    ACTIVE = "active"
    INACTIVE = "inactive"
    STARTING = "starting"
    STOPPING = "stopping"
    LOADING = "loading"


_ALLOWED = {
    (ModelStatus.STOPPING, ModelStatus.INACTIVE), (ModelStatus.STARTING, ModelStatus.INACTIVE),
    (ModelStatus.INACTIVE, ModelStatus.STARTING), (ModelStatus.STARTING, ModelStatus.ACTIVE),
    (ModelStatus.STOPPING, ModelStatus.ACTIVE), (ModelStatus.INACTIVE, ModelStatus.ACTIVE),
}


def valid_transition(a: ModelStatus, b: ModelStatus) -> bool:
    return a == b or b == ModelStatus.STOPPING or (a, b) in _ALLOWED


@dataclass
class ModelInfo:
    id: int
    name: str
    version: str = "1.0"
    framework: str = "llm"
    device: str = "cuda:0"
    optimization_level: str = "default"
    model_path: str = ""
    status: ModelStatus = ModelStatus.ACTIVE
    replica_id: int = 0
    base_model_id: Optional[int] = None
    loaded_at: int = field(default_factory=lambda: int(time.time()))

    def __post_init__(self):
        if self.base_model_id is None:
            self.base_model_id = self.id


@dataclass
class ModelMetric:
    latencies_ms: list = field(default_factory=list)
    requests: int = 0
    errors: int = 0

    def percentile(self, q: float) -> float:
        if not self.latencies_ms:
            return 0.0
        s = sorted(self.latencies_ms)
        return s[min(len(s) - 1, int(round(q / 100.0 * (len(s) - 1))))]


class ModelRegistry:
    MAX_SAMPLES = 10_000

    def __init__(self):
        self._models: dict = {}
        self._history: dict = {}
        self._metrics: dict = {}
        self._listeners: list = []
        self._lock = threading.RLock()

    def add_listener(self, fn: Callable) -> None:
        self._listeners.append(fn)

    def _emit(self, *event) -> None:
        for fn in self._listeners:
            fn(*event)

    def register(self, info: ModelInfo) -> None:
        with self._lock:
            self._models[info.id] = info
            self._history[info.id] = [info.status]
            self._metrics[info.id] = ModelMetric()
        self._emit("registered", info.id)

    def unregister(self, model_id: int) -> Optional[ModelInfo]:
        with self._lock:
            info = self._models.pop(model_id, None)
            self._history.pop(model_id, None)
            self._metrics.pop(model_id, None)
        if info is not None:
            self._emit("unregistered", model_id)
        return info

    def get(self, model_id: int) -> Optional[ModelInfo]:
        return self._models.get(model_id)

    def list(self) -> list:
        return sorted(self._models.values(), key=lambda m: m.id)

    def replicas_of(self, base_model_id: int) -> list:
        return [m for m in self.list() if m.base_model_id == base_model_id]

    def next_id(self) -> int:
        return max(self._models, default=0) + 1

    def update_status(self, model_id: int, status: ModelStatus) -> bool:
        with self._lock:
            info = self._models.get(model_id)
            if info is None or not valid_transition(info.status, status):
                return False
            old = info.status
            info.status = status
            self._history[model_id].append(status)
        self._emit("status_changed", model_id, old, status)
        return True

    def status_history(self, model_id: int) -> list:
        return list(self._history.get(model_id, []))

    def rollback_status(self, model_id: int) -> Optional[ModelStatus]:
        """Return to the previous status (if that transition is valid)."""
        with self._lock:
            h = self._history.get(model_id)
            info = self._models.get(model_id)
            if not h or len(h) < 2 or info is None:
                return None
            prev = h[-2]
            if not valid_transition(info.status, prev):
                return None
            h.pop()
            info.status = prev
        self._emit("status_changed", model_id, None, prev)
        return prev

    def record_latency(self, model_id: int, ms: float, ok: bool = True) -> None:
        m = self._metrics.get(model_id)
        if m is None:
            return
        m.requests += 1
        if not ok:
            m.errors += 1
        m.latencies_ms.append(ms)
        if len(m.latencies_ms) > self.MAX_SAMPLES:
            del m.latencies_ms[: len(m.latencies_ms) - self.MAX_SAMPLES]

    def latency_summary(self, model_id: int) -> dict:
        m = self._metrics.get(model_id) or ModelMetric()
        return {"p50": m.percentile(50), "p95": m.percentile(95), "p99": m.percentile(99),
                "requests": m.requests, "errors": m.errors}
