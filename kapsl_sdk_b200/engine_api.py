"""Engine API (L4): request/response types, error taxonomy and the Engine interface.

Mirrors crates/kapsl-engine-api/src/lib.rs: ``EngineError`` variants and their
display strings (lib.rs:14-61, sent verbatim in ERR frames), ``EngineMetrics``
(130-188), ``TensorDtype`` string names and aliases (190-270),
``BinaryTensorPacket`` with byte-length validation (272-460),
``RequestMetadata`` (462-492), ``InferenceRequest`` (494-567),
``CancellationToken`` (500-519), ``EngineModelInfo`` (569-585) and the
``Engine`` trait (587-728).  The bincode encoding of these types lives in the
C++ wire codec (``kapsl_sdk_b200._native``) with a Python mirror in
:mod:`kapsl_sdk_b200.server.wire`.
"""
from __future__ import annotations

import abc
import enum
import threading
import time
from dataclasses import dataclass, field
from typing import Iterator, Optional

import numpy as np


class ErrorKind(enum.Enum):
    BACKEND = "Backend error: {}"
    INVALID_INPUT = "Invalid input: {}"
    MODEL_NOT_LOADED = "Model not loaded"
    OVERLOADED = "System overloaded: {}"
    MODEL_LOAD = "Model load error for {}"
    INFERENCE = "Inference error: {}"
    TIMEOUT = "Timeout: {}"
    RESOURCE_EXHAUSTED = "Resource exhausted: {}"
    CANCELLED = "Cancelled: {}"


class EngineError(Exception):
    """Engine failure; ``str()`` gives the reference's display string."""

    def __init__(self, kind: ErrorKind, message: str = ""):
        self.kind = kind
        self.message = message
        super().__init__(str(self))

    def __str__(self) -> str:
        if self.kind is ErrorKind.MODEL_NOT_LOADED:
            return self.kind.value
        return self.kind.value.format(self.message)

    @classmethod
    def backend(cls, m: str) -> "EngineError":
        return cls(ErrorKind.BACKEND, m)

    @classmethod
    def invalid_input(cls, m: str) -> "EngineError":
        return cls(ErrorKind.INVALID_INPUT, m)

    @classmethod
    def model_not_loaded(cls) -> "EngineError":
        return cls(ErrorKind.MODEL_NOT_LOADED)

    @classmethod
    def overloaded(cls, m: str) -> "EngineError":
        return cls(ErrorKind.OVERLOADED, m)

    @classmethod
    def model_load(cls, path: str, source: str) -> "EngineError":
        return cls(ErrorKind.MODEL_LOAD, f"{path}: {source}")

    @classmethod
    def inference(cls, m: str) -> "EngineError":
        return cls(ErrorKind.INFERENCE, m)

    @classmethod
    def timeout(cls, m: str) -> "EngineError":
        return cls(ErrorKind.TIMEOUT, m)

    @classmethod
    def resource_exhausted(cls, m: str) -> "EngineError":
        return cls(ErrorKind.RESOURCE_EXHAUSTED, m)

    @classmethod
    def cancelled(cls, m: str) -> "EngineError":
        return cls(ErrorKind.CANCELLED, m)

    @property
    def is_overloaded(self) -> bool:
        return self.kind is ErrorKind.OVERLOADED


class TensorDtype(enum.Enum):
    FLOAT32 = "float32"
    FLOAT64 = "float64"
    FLOAT16 = "float16"
    INT32 = "int32"
    INT64 = "int64"
    UINT8 = "uint8"
    UTF8 = "string"

    @classmethod
    def parse(cls, s: str) -> "TensorDtype":
        key = s.strip().lower()
        aliases = {"float32": "float32", "fp32": "float32", "f32": "float32", "float64": "float64",
                   "fp64": "float64", "f64": "float64", "float16": "float16", "fp16": "float16", "f16": "float16",
                   "int32": "int32", "i32": "int32", "int64": "int64", "i64": "int64", "uint8": "uint8",
                   "u8": "uint8", "string": "string", "utf8": "string", "str": "string"}
        if key not in aliases:
            raise EngineError.invalid_input(f"Unsupported dtype: {s}")
        return cls(aliases[key])

    def as_str(self) -> str:
        return self.value

    @property
    def itemsize(self) -> int:
        return {"float32": 4, "float64": 8, "float16": 2, "int32": 4, "int64": 8, "uint8": 1, "string": 1}[self.value]

    def numpy(self):
        return {"float32": np.float32, "float64": np.float64, "float16": np.float16, "int32": np.int32,
                "int64": np.int64, "uint8": np.uint8, "string": np.uint8}[self.value]


@dataclass
class BinaryTensorPacket:
    shape: list
    dtype: TensorDtype
    data: bytes

    def validate(self) -> None:
        """Dimensions must be > 0 and the byte length must match (string: any length)."""
        for d in self.shape:
            if d <= 0:
                raise EngineError.invalid_input(f"Invalid tensor dimension {d} in shape {self.shape}")
        if self.dtype is TensorDtype.UTF8:
            return
        n = 1
        for d in self.shape:
            n *= d
        want = n * self.dtype.itemsize
        if len(self.data) != want:
            raise EngineError.invalid_input(
                f"Data size mismatch: expected {want} bytes for shape {self.shape} ({self.dtype.as_str()}), "
                f"got {len(self.data)}")

    def to_numpy(self) -> np.ndarray:
        if self.dtype is TensorDtype.UTF8:
            raise EngineError.invalid_input("string tensors have no numeric view")
        return np.frombuffer(self.data, dtype=self.dtype.numpy()).reshape(self.shape)

    def text(self) -> str:
        return self.data.decode("utf-8", errors="replace")

    @classmethod
    def from_numpy(cls, a: np.ndarray) -> "BinaryTensorPacket":
        m = {np.dtype(np.float32): TensorDtype.FLOAT32, np.dtype(np.float64): TensorDtype.FLOAT64,
             np.dtype(np.float16): TensorDtype.FLOAT16, np.dtype(np.int32): TensorDtype.INT32,
             np.dtype(np.int64): TensorDtype.INT64, np.dtype(np.uint8): TensorDtype.UINT8}
        a = np.ascontiguousarray(a)
        return cls(list(a.shape), m[a.dtype], a.tobytes())

    @classmethod
    def from_text(cls, s: str) -> "BinaryTensorPacket":
        b = s.encode("utf-8")
        return cls([1, max(len(b), 1)], TensorDtype.UTF8, b)


@dataclass
class NamedTensor:
    name: str
    tensor: BinaryTensorPacket


@dataclass
class RequestMetadata:
    request_id: Optional[str] = None
    timeout_ms: Optional[int] = None
    priority: Optional[int] = None
    force_cpu: Optional[bool] = None
    model_version: Optional[str] = None
    auth_token: Optional[str] = None
    max_new_tokens: Optional[int] = None
    temperature: Optional[float] = None
    top_p: Optional[float] = None
    top_k: Optional[int] = None
    repetition_penalty: Optional[float] = None
    seed: Optional[int] = None
    stop_token_ids: Optional[list] = None


class CancellationToken:
    def __init__(self):
        self._ev = threading.Event()

    def cancel(self) -> None:
        self._ev.set()

    def is_cancelled(self) -> bool:
        return self._ev.is_set()


@dataclass
class InferenceRequest:
    input: BinaryTensorPacket
    additional_inputs: list = field(default_factory=list)
    session_id: Optional[str] = None
    metadata: Optional[RequestMetadata] = None
    cancellation: Optional[CancellationToken] = None  # not on the wire

    @property
    def request_id(self) -> Optional[str]:
        return self.metadata.request_id if self.metadata else None


@dataclass
class EngineMetrics:
    inference_time: float = 0.0
    memory_usage: int = 0
    gpu_utilization: float = 0.0
    throughput: float = 0.0
    batch_size: int = 0
    queue_depth: int = 0
    error_rate: float = 0.0
    collected_at_ms: int = field(default_factory=lambda: int(time.time() * 1000))
    kv_cache_bytes_used: int = 0
    kv_cache_bytes_capacity: int = 0
    kv_cache_blocks_total: int = 0
    kv_cache_blocks_free: int = 0
    kv_cache_sequences: int = 0
    kv_cache_evicted_blocks: int = 0
    kv_cache_evicted_sequences: int = 0
    kv_cache_packed_layers: int = 0


@dataclass
class EngineModelInfo:
    input_names: list = field(default_factory=list)
    output_names: list = field(default_factory=list)
    input_shapes: list = field(default_factory=list)
    output_shapes: list = field(default_factory=list)
    input_dtypes: list = field(default_factory=list)
    output_dtypes: list = field(default_factory=list)
    framework: Optional[str] = None
    model_version: Optional[str] = None
    peak_concurrency: Optional[int] = None


class Engine(abc.ABC):
    """Serving interface every backend implements (reference ``Engine`` trait)."""

    @abc.abstractmethod
    def load(self, model_path: str) -> None: ...

    @abc.abstractmethod
    def infer(self, request: InferenceRequest) -> BinaryTensorPacket: ...

    def infer_async(self, request: InferenceRequest):
        """Run ``infer`` on a worker thread; returns a ``concurrent.futures.Future``."""
        import concurrent.futures as cf

        ex = cf.ThreadPoolExecutor(max_workers=1)
        fut = ex.submit(self.infer, request)
        ex.shutdown(wait=False)
        return fut

    def infer_batch(self, requests: list) -> list:
        """Default: one ``infer`` per request (reference default loops too)."""
        return [self.infer(r) for r in requests]

    def infer_stream(self, request: InferenceRequest) -> Iterator[BinaryTensorPacket]:
        """Default: a single-item stream."""
        yield self.infer(request)

    def infer_with_cancellation(self, request: InferenceRequest) -> BinaryTensorPacket:
        tok = request.cancellation
        if tok is not None and tok.is_cancelled():
            raise EngineError.cancelled("request cancelled before execution")
        out = self.infer(request)
        if tok is not None and tok.is_cancelled():
            raise EngineError.cancelled("request cancelled during execution")
        return out

    def warmup(self) -> None:
        return None

    def unload(self) -> None:
        return None

    def metrics(self) -> EngineMetrics:
        return EngineMetrics()

    def model_info(self) -> EngineModelInfo:
        return EngineModelInfo()

    def health_check(self) -> bool:
        return True
