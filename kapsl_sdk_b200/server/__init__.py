"""Serving front-end: Unix-socket, TCP and shared-memory servers.

``KapslServer`` wires the native servers (``kapsl_sdk_b200._native``) to a
model table.  Defaults match the reference runtime: Unix socket
``/tmp/kapsl.sock``, TCP ``127.0.0.1:9096``, SHM name ``kapsl-shm-default``.
"""
from __future__ import annotations

from typing import Optional

from .dispatch import Dispatcher, EngineTarget

DEFAULT_SOCKET = "/tmp/kapsl.sock"
DEFAULT_TCP_PORT = 9096
DEFAULT_SHM_NAME = "kapsl-shm-default"


def _peak_concurrency(target) -> int:
    eng = getattr(target, "engine", target)
    try:
        v = eng.model_info().peak_concurrency if hasattr(eng, "model_info") else None
    except Exception:
        v = None
    v = v or getattr(target, "peak_concurrency", None) or 1
    return min(max(int(v), 1), 1000)


class KapslServer:
    def __init__(self, models: Optional[dict] = None, lookup=None, api_token: Optional[str] = None):
        """``models`` maps model id -> target (object with infer/infer_stream, or an
        Engine which is wrapped); or pass ``lookup(model_id)`` directly."""
        from .._ext import native

        self.models = {}
        for k, v in (models or {}).items():
            self.add_model(k, v)
        self._lookup = lookup or self.models.get
        self.dispatcher = Dispatcher(self._lookup)
        self.api_token = api_token
        self._native = native()
        self.wire = self._native.WireServer(self.dispatcher, api_token)
        self.shm = None
        self.tcp_port = None
        self.socket_path = None

    def add_model(self, model_id: int, target) -> None:
        if not hasattr(target, "infer_stream") or not hasattr(target, "infer"):
            raise TypeError("target needs infer() and infer_stream()")
        from ..engine_api import Engine

        self.models[int(model_id)] = EngineTarget(target) if isinstance(target, Engine) else target

    def listen_unix(self, path: str = DEFAULT_SOCKET) -> "KapslServer":
        self.wire.listen_unix(path)
        self.socket_path = path
        return self

    def listen_tcp(self, host: str = "127.0.0.1", port: int = DEFAULT_TCP_PORT) -> "KapslServer":
        self.tcp_port = self.wire.listen_tcp(host, port)
        return self

    def serve_shm(self, name: str = DEFAULT_SHM_NAME, size: int = 256 << 20, workers: int = 4,
                  model_weights: Optional[dict] = None) -> "KapslServer":
        """Result slots come from one sub-pool per model, sized in proportion to
        ``model_weights`` (model id -> expected concurrency; by default each
        model's ``peak_concurrency`` from ``model_info()`` or as an attribute,
        else 1), plus a shared overflow
        pool of 10% that also serves unknown model ids."""
        if model_weights is None:
            model_weights = {mid: _peak_concurrency(t) for mid, t in self.models.items()}
        self.shm = self._native.ShmServer(self.dispatcher, name, size, workers,
                                          {int(k): max(1, int(v)) for k, v in model_weights.items()})
        self.wire.attach_shm(name)  # hybrid requests read/write the same region
        return self

    def start(self) -> "KapslServer":
        self.wire.start()
        if self.shm is not None:
            self.shm.start()
        return self

    def stop(self) -> None:
        if self.shm is not None:
            self.shm.stop()
        self.wire.stop()

    def __enter__(self):
        return self.start()

    def __exit__(self, *a):
        self.stop()
