"""Prometheus metrics and the monitoring middleware
(crates/kapsl-monitor/src/metrics.rs:5-234, middleware.rs:14-329).

Metric names and labels are the reference's:
``kapsl_inference_latency_seconds{model,version,status}`` (buckets 1 ms .. 5 s),
``kapsl_inference_total{model,status}``, ``kapsl_active_inferences``,
``kapsl_batch_size``, ``kapsl_queue_wait_seconds``,
``kapsl_pool_{active_replicas,queue_depth_high,queue_depth_low,healthy_replicas}``,
``kapsl_kv_cache_{bytes_used,bytes_capacity,blocks_total,blocks_free,sequences,
evicted_blocks_total,evicted_sequences_total,packed_layers}`` and the SHM pool
gauges ``kapsl_shm_pool_{in_use,exhausted_total,oldest_lease_ms}``; added for the
LLM serving metrics: ``kapsl_ttft_seconds``, ``kapsl_tpot_seconds``,
``kapsl_output_tokens_total``.

``MonitoringMiddleware`` wraps any Engine, times and counts requests, takes the
batch size from ``shape[0]`` and estimates peak concurrency as the p95 of
sampled in-flight counts over a window (``KAPSL_PEAK_CONCURRENCY_WINDOW``,
``KAPSL_PEAK_CONCURRENCY_SAMPLE_STRIDE``), reported via ``model_info()``.
"""
from __future__ import annotations

import os
import threading
import time
from typing import Optional

from ..engine_api import Engine, EngineError, EngineMetrics, EngineModelInfo, InferenceRequest

LATENCY_BUCKETS = (0.001, 0.0025, 0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0)


class KapslMetrics:
    def __init__(self, registry=None):
        from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram

        self.registry = registry or CollectorRegistry()
        r = self.registry
        self.latency = Histogram("kapsl_inference_latency_seconds", "Inference latency", ["model", "version", "status"],
                                 buckets=LATENCY_BUCKETS, registry=r)
        self.total = Counter("kapsl_inference", "Inference requests", ["model", "status"], registry=r)
        self.active = Gauge("kapsl_active_inferences", "In-flight inferences", ["model"], registry=r)
        self.batch = Histogram("kapsl_batch_size", "Batch size", ["model"], buckets=(1, 2, 4, 8, 16, 32, 64, 128),
                               registry=r)
        self.queue_wait = Histogram("kapsl_queue_wait_seconds", "Queue wait", ["model"], buckets=LATENCY_BUCKETS,
                                    registry=r)
        self.pool = {k: Gauge(f"kapsl_pool_{k}", k.replace("_", " "), ["model"], registry=r)
                     for k in ("active_replicas", "queue_depth_high", "queue_depth_low", "healthy_replicas")}
        kv = ("bytes_used", "bytes_capacity", "blocks_total", "blocks_free", "sequences", "evicted_blocks_total",
              "evicted_sequences_total", "packed_layers")
        self.kv = {k: Gauge(f"kapsl_kv_cache_{k}", k.replace("_", " "), ["model"], registry=r) for k in kv}
        self.shm = {k: Gauge(f"kapsl_shm_pool_{k}", k.replace("_", " "), registry=r)
                    for k in ("in_use", "exhausted_total", "oldest_lease_ms")}
        self.ttft = Histogram("kapsl_ttft_seconds", "Time to first token", ["model"], buckets=LATENCY_BUCKETS,
                              registry=r)
        self.tpot = Histogram("kapsl_tpot_seconds", "Time per output token", ["model"], buckets=LATENCY_BUCKETS,
                              registry=r)
        self.out_tokens = Counter("kapsl_output_tokens", "Generated tokens", ["model"], registry=r)

    def update_engine(self, model: str, m: EngineMetrics) -> None:
        self.kv["bytes_used"].labels(model).set(m.kv_cache_bytes_used)
        self.kv["bytes_capacity"].labels(model).set(m.kv_cache_bytes_capacity)
        self.kv["blocks_total"].labels(model).set(m.kv_cache_blocks_total)
        self.kv["blocks_free"].labels(model).set(m.kv_cache_blocks_free)
        self.kv["sequences"].labels(model).set(m.kv_cache_sequences)
        self.kv["evicted_blocks_total"].labels(model).set(m.kv_cache_evicted_blocks)
        self.kv["evicted_sequences_total"].labels(model).set(m.kv_cache_evicted_sequences)
        self.kv["packed_layers"].labels(model).set(m.kv_cache_packed_layers)

    def update_pool(self, model: str, pool) -> None:
        h, l = pool.get_queue_depth()
        self.pool["active_replicas"].labels(model).set(pool.size())
        self.pool["healthy_replicas"].labels(model).set(pool.healthy_count())
        self.pool["queue_depth_high"].labels(model).set(h)
        self.pool["queue_depth_low"].labels(model).set(l)

    def update_shm(self, server) -> None:
        self.shm["in_use"].set(server.pool_in_use)
        self.shm["exhausted_total"].set(server.pool_exhausted)
        self.shm["oldest_lease_ms"].set(server.pool_oldest_lease_ms)

    def exposition(self) -> bytes:
        from prometheus_client import generate_latest

        return generate_latest(self.registry)


def serve_metrics(metrics: KapslMetrics, port: int = 9100, addr: str = "127.0.0.1"):
    """Expose ``metrics`` over HTTP (``GET /metrics``, Prometheus text format) from a
    daemon thread; returns the HTTP server (``shutdown()`` to stop).  The reference
    registers the same metrics but ships no exporter."""
    from prometheus_client import start_http_server

    server, _thread = start_http_server(port, addr=addr, registry=metrics.registry)
    return server


class MonitoringMiddleware(Engine):
    def __init__(self, inner: Engine, metrics: KapslMetrics, model: str = "model", version: str = "1"):
        self.inner = inner
        self.m = metrics
        self.model = model
        self.version = version
        self._active = 0
        self._lock = threading.Lock()
        self.window = int(os.environ.get("KAPSL_PEAK_CONCURRENCY_WINDOW", "512"))
        self.stride = max(1, int(os.environ.get("KAPSL_PEAK_CONCURRENCY_SAMPLE_STRIDE", "1")))
        self._samples: list = []
        self._n = 0

    def _enter(self) -> None:
        with self._lock:
            self._active += 1
            self._n += 1
            if self._n % self.stride == 0:
                self._samples.append(self._active)
                if len(self._samples) > self.window:
                    self._samples.pop(0)
        self.m.active.labels(self.model).inc()

    def _exit(self) -> None:
        with self._lock:
            self._active -= 1
        self.m.active.labels(self.model).dec()

    def peak_concurrency(self) -> int:
        with self._lock:
            s = sorted(self._samples)
        if not s:
            return 1
        return max(1, s[min(len(s) - 1, int(0.95 * (len(s) - 1) + 0.5))])

    def load(self, model_path: str) -> None:
        self.inner.load(model_path)

    def infer(self, request: InferenceRequest):
        self._enter()
        t0 = time.perf_counter()
        status = "success"
        try:
            if request.input.shape:
                self.m.batch.labels(self.model).observe(max(1, request.input.shape[0]))
            return self.inner.infer(request)
        except Exception:
            status = "error"
            raise
        finally:
            self.m.latency.labels(self.model, self.version, status).observe(time.perf_counter() - t0)
            self.m.total.labels(self.model, status).inc()
            self._exit()

    def infer_stream(self, request: InferenceRequest):
        self._enter()
        t0 = time.perf_counter()
        try:
            it = self.inner.infer_stream(request)
        except Exception:
            self.m.total.labels(self.model, "error").inc()
            self._exit()
            raise

        def gen():
            status = "success"
            first = None
            n = 0
            try:
                for pkt in it:
                    now = time.perf_counter()
                    if first is None:
                        first = now
                        self.m.ttft.labels(self.model).observe(now - t0)
                    n += 1
                    yield pkt
            except Exception:
                status = "error"
                raise
            finally:
                end = time.perf_counter()
                if first is not None and n > 1:
                    self.m.tpot.labels(self.model).observe((end - first) / (n - 1))
                self.m.out_tokens.labels(self.model).inc(n)
                self.m.latency.labels(self.model, self.version, status).observe(end - t0)
                self.m.total.labels(self.model, status).inc()
                self._exit()

        return gen()

    def metrics(self) -> EngineMetrics:
        em = self.inner.metrics()
        self.m.update_engine(self.model, em)
        return em

    def model_info(self) -> EngineModelInfo:
        info = self.inner.model_info()
        info.peak_concurrency = self.peak_concurrency()
        return info

    def health_check(self) -> bool:
        return self.inner.health_check()

    def unload(self) -> None:
        self.inner.unload()
