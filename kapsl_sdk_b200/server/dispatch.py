"""Python side of the native servers: turns decoded wire requests into
engine calls.

The C++ ``WireServer`` / ``ShmServer`` own the sockets, framing, bincode and
auth; for each request they call ``Dispatcher.infer`` or
``Dispatcher.infer_stream`` with the decoded request as a dict.  The
dispatcher resolves ``model_id`` to a scheduler (reference:
``SchedulerLookup = Fn(u32) -> Option<Arc<dyn ReplicaScheduler>>``,
crates/kapsl-ipc/src/server.rs:24-25) and converts packets both ways.
Unknown ids raise ``Model {id} not found`` (server.rs:266, 447).
"""
from __future__ import annotations

from typing import Callable, Iterator, Optional

from ..engine_api import (BinaryTensorPacket, EngineError, InferenceRequest, NamedTensor, RequestMetadata,
                          TensorDtype)


def packet_from_tuple(t) -> BinaryTensorPacket:
    shape, dtype, data = t
    return BinaryTensorPacket(list(shape), TensorDtype.parse(dtype), bytes(data))


def packet_to_tuple(p: BinaryTensorPacket) -> tuple:
    return (list(p.shape), p.dtype.as_str(), bytes(p.data))


def request_from_dict(d: dict) -> InferenceRequest:
    md = d.get("metadata")
    meta = RequestMetadata(**md) if md else None
    return InferenceRequest(
        input=packet_from_tuple(d["input"]),
        additional_inputs=[NamedTensor(n, packet_from_tuple(p)) for n, p in d.get("additional_inputs") or []],
        session_id=d.get("session_id"),
        metadata=meta,
    )


class Dispatcher:
    """``lookup(model_id)`` returns an object with ``infer(request, priority)``
    and ``infer_stream(request)`` (a ReplicaPool, Scheduler or Engine adapter)."""

    def __init__(self, lookup: Callable[[int], Optional[object]]):
        self.lookup = lookup

    def _target(self, model_id: int):
        t = self.lookup(int(model_id))
        if t is None:
            raise RuntimeError(f"Model {model_id} not found")
        return t

    def infer(self, model_id: int, req: dict, priority: str) -> tuple:
        target = self._target(model_id)
        request = request_from_dict(req)
        out = target.infer(request, priority=priority)
        return packet_to_tuple(out)

    def infer_stream(self, model_id: int, req: dict) -> Iterator[tuple]:
        target = self._target(model_id)
        request = request_from_dict(req)
        native = getattr(target, "infer_stream_native", None)
        if native is not None:
            # a token-id stream the native server writes without the GIL (None: not
            # applicable to this request, take the packet iterator)
            ch = native(request)
            if ch is not None:
                return ch
        stream = target.infer_stream(request)  # errors here are "initial" failures

        def gen():
            try:
                for pkt in stream:
                    yield packet_to_tuple(pkt)
            finally:
                close = getattr(stream, "close", None)
                if close is not None:
                    close()

        return gen()


class EngineTarget:
    """Adapts a bare :class:`~kapsl_sdk_b200.engine_api.Engine` to the dispatcher."""

    def __init__(self, engine):
        self.engine = engine

    def infer(self, request: InferenceRequest, priority: str = "throughput") -> BinaryTensorPacket:
        return self.engine.infer(request)

    def infer_stream(self, request: InferenceRequest):
        return self.engine.infer_stream(request)

    def infer_stream_native(self, request: InferenceRequest):
        native = getattr(self.engine, "infer_stream_native", None)
        return native(request) if native is not None else None
