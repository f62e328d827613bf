"""Rank liveness for multi-process serving.

Every rank runs a :class:`HeartbeatMonitor`: a daemon thread writes the
rank's wall-clock time into the torch.distributed key-value store every
``interval_s`` and reads the other ranks' entries.  A rank whose entry is
older than ``timeout_s`` (or never appeared within ``timeout_s`` of start)
is reported dead; ``check()`` raises :class:`RankFailure` naming it.  The
serving loops call ``check()`` between steps, so a peer that crashed or
hangs is detected on the host before the next collective or peer-memory
kernel is launched (the kernels' own waits are bounded as well, so a lost
peer never hangs a GPU).  Combined with a short process-group timeout this
turns a lost rank into an exception on every survivor.

The reference has no cross-process failure detection (its health checks are
per engine: crates/kapsl-backends/src/engine_pool.rs:121-194).
"""
from __future__ import annotations

import threading
import time
from typing import Optional


class RankFailure(RuntimeError):
    def __init__(self, ranks: list, detail: str = ""):
        super().__init__(f"rank(s) {ranks} stopped responding{': ' + detail if detail else ''}")
        self.ranks = ranks


class HeartbeatMonitor:
    def __init__(self, store, rank: int, world: int, interval_s: float = 0.5, timeout_s: float = 5.0,
                 prefix: str = "kapsl/hb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval_s, self.timeout_s, self.prefix = interval_s, timeout_s, prefix
        self._stop = threading.Event()
        self._dead: list = []
        self._lock = threading.Lock()
        self._t0 = time.time()
        self._thread: Optional[threading.Thread] = None

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def start(self) -> "HeartbeatMonitor":
        self._beat()
        self._thread = threading.Thread(target=self._run, name="kapsl-heartbeat", daemon=True)
        self._thread.start()
        return self

    def _beat(self) -> None:
        self.store.set(self._key(self.rank), repr(time.time()))

    def _scan(self) -> list:
        now = time.time()
        dead = []
        for r in range(self.world):
            if r == self.rank:
                continue
            k = self._key(r)
            if not self.store.check([k]):
                if now - self._t0 > self.timeout_s:
                    dead.append(r)
                continue
            try:
                last = float(self.store.get(k))
            except Exception:
                continue
            if now - last > self.timeout_s:
                dead.append(r)
        return dead

    def _run(self) -> None:
        while not self._stop.wait(self.interval_s):
            try:
                self._beat()
                dead = self._scan()
            except Exception:  # the store itself is gone (rank 0 died): everyone is cut off
                dead = [0] if self.rank != 0 else []
            with self._lock:
                self._dead = dead

    def dead_ranks(self) -> list:
        with self._lock:
            return list(self._dead)

    def check(self) -> None:
        dead = self.dead_ranks()
        if dead:
            raise RankFailure(dead)

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2 * self.interval_s + 1)


def init_distributed(backend: str, timeout_s: float = 120.0, device=None):
    """``torch.distributed.init_process_group`` for serving groups, with the NCCL
    watchdog configured to abort: ``TORCH_NCCL_ASYNC_ERROR_HANDLING=1`` makes the
    process group's watchdog thread poll each communicator's asynchronous error
    state and abort the communicators of a collective that failed or outlived
    ``timeout_s``, so the waiting ranks get an exception instead of blocking (the
    reference's plan of non-blocking communicators polled for async errors and
    aborted on timeout).  A value already in the environment is kept."""
    import os
    from datetime import timedelta

    import torch.distributed as dist

    if backend == "nccl":
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    kw = {"timeout": timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
