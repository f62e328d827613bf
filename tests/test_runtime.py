"""Control plane: priority, request scheduler, replica pool, router, autoscaler,
registry, cron, device preference, mesh/collectives, monitoring, engine pool,
backend factory.  Behaviours follow the reference's unit tests."""
import threading
import time

import numpy as np
import pytest

from kapsl_sdk_b200.engine_api import (BinaryTensorPacket, CancellationToken, Engine, EngineError, EngineMetrics,
                                       InferenceRequest, RequestMetadata, TensorDtype)
from kapsl_sdk_b200.runtime.scheduler import (OverflowPolicy, Priority, SchedMetadata, Scheduler,
                                              determine_priority)


def pkt(b=b"x"):
    return BinaryTensorPacket([len(b)], TensorDtype.UINT8, b)


class Echo(Engine):
    def __init__(self, delay=0.0, fail=False, kv=None):
        self.delay, self.fail, self.kv = delay, fail, kv
        self.batches = []

    def load(self, p):
        pass

    def infer(self, r):
        if self.fail:
            raise EngineError.backend("replica down")
        time.sleep(self.delay)
        return r.input

    def infer_batch(self, rs):
        self.batches.append(len(rs))
        return [self.infer(r) for r in rs]

    def infer_stream(self, r):
        if self.fail:
            raise EngineError.backend("replica down")
        return iter([r.input])

    def metrics(self):
        m = EngineMetrics()
        if self.kv:
            m.kv_cache_blocks_total, m.kv_cache_blocks_free = self.kv
            m.kv_cache_bytes_capacity = self.kv[0] * 100
            m.kv_cache_bytes_used = (self.kv[0] - self.kv[1]) * 100
        return m


def test_priority_heuristics():
    assert determine_priority(SchedMetadata(priority=0, batch_size=100)) is Priority.LATENCY_CRITICAL
    assert determine_priority(SchedMetadata(sla_deadline_ms=100, batch_size=100)) is Priority.LATENCY_CRITICAL
    assert determine_priority(SchedMetadata(input_size_bytes=1000, batch_size=100)) is Priority.LATENCY_CRITICAL
    assert determine_priority(SchedMetadata(batch_size=3)) is Priority.LATENCY_CRITICAL
    assert determine_priority(SchedMetadata(batch_size=16, input_size_bytes=10_000_000)) is Priority.THROUGHPUT


def test_scheduler_microbatches_low_priority():
    eng = Echo(delay=0.01)
    s = Scheduler([eng], max_micro_batch=8, queue_delay_ms=20)
    try:
        outs = []
        ts = [threading.Thread(target=lambda i=i: outs.append(s.infer(InferenceRequest(pkt(bytes([i])))))) for i in
              range(8)]
        [t.start() for t in ts]
        [t.join() for t in ts]
        assert len(outs) == 8 and max(eng.batches) > 1
        assert s.infer(InferenceRequest(pkt(b"h")), Priority.LATENCY_CRITICAL).data == b"h"
    finally:
        s.shutdown()


def test_scheduler_overflow_and_health():
    eng = Echo(delay=0.2)
    s = Scheduler([eng], queue_size=2, overflow=OverflowPolicy.DROP_NEWEST, max_micro_batch=1)
    try:
        futs = []
        with pytest.raises(EngineError):
            for _ in range(10):
                futs.append(s.try_infer(InferenceRequest(pkt())))
        assert not s.is_healthy()
        for f in futs:
            f.result(timeout=5)
        assert s.is_healthy()
    finally:
        s.shutdown()


def test_scheduler_cancellation_and_force_cpu():
    eng, cpu = Echo(delay=0.05), Echo()
    s = Scheduler([eng], cpu_engine=cpu, max_micro_batch=1)
    try:
        tok = CancellationToken()
        tok.cancel()
        with pytest.raises(EngineError, match="Cancelled"):
            s.infer(InferenceRequest(pkt(), cancellation=tok))
        r = InferenceRequest(pkt(b"c"), metadata=RequestMetadata(force_cpu=True))
        assert s.infer(r).data == b"c"
    finally:
        s.shutdown()


def test_replica_pool_failover_and_kv_aware_routing():
    from kapsl_sdk_b200.runtime.replica_pool import PoolStrategy, ReplicaPool

    bad, good = Scheduler([Echo(fail=True)]), Scheduler([Echo()])
    pool = ReplicaPool(PoolStrategy.ROUND_ROBIN)
    pool.add_replica(0, bad)
    pool.add_replica(1, good)
    try:
        assert pool.infer(InferenceRequest(pkt(b"f"))).data == b"f"
        assert list(pool.infer_stream(InferenceRequest(pkt(b"s"))))[0].data == b"s"
        assert pool.stats()[1].requests_total >= 1
        # least loaded prefers the replica with KV headroom (tier 0 vs tier 3)
        full, roomy = Scheduler([Echo(kv=(100, 2))]), Scheduler([Echo(kv=(100, 90))])
        p2 = ReplicaPool(PoolStrategy.LEAST_LOADED)
        p2.add_replica(0, full)
        p2.add_replica(1, roomy)
        order = p2._ordered(InferenceRequest(pkt()))
        assert order[0].replica_id == 1
        # sticky: same session -> same replica
        p3 = ReplicaPool(PoolStrategy.STICKY)
        for i in range(4):
            p3.add_replica(i, Scheduler([Echo()]))
        firsts = {p3._ordered(InferenceRequest(pkt(), session_id="abc"))[0].replica_id for _ in range(5)}
        assert len(firsts) == 1
        assert pool.remove_replica(0) and pool.size() == 1
    finally:
        for x in (bad, good):
            x.shutdown()


def test_router():
    from kapsl_sdk_b200.runtime.router import MeshRouter

    r = MeshRouter.round_robin(3)
    assert [r.route() for _ in range(4)] == [0, 1, 2, 0]
    assert r.route("s1") == r.route("s1")
    tp = MeshRouter.tensor_parallel(8, 4)
    assert {tp.route() for _ in range(4)} == {0, 4}
    assert MeshRouter.pipeline(4).route("x") == 0


def test_autoscaler_hysteresis_and_cooldown():
    from kapsl_sdk_b200.runtime.autoscaler import AutoScaler, ScalingPolicy

    now = [1000.0]
    a = AutoScaler(clock=lambda: now[0])
    a.register_policy(1, ScalingPolicy(min_replicas=1, max_replicas=3, target_queue_depth=5, scale_down_threshold=2,
                                       cooldown_seconds=60))
    assert a.should_scale_up(1, 1, 1, 50, 10.0) is None        # below 20 s hysteresis
    assert a.should_scale_up(1, 1, 1, 50, 10.0) == 2           # +1 step only
    assert a.should_scale_up(1, 2, 1, 50, 30.0) is None        # degraded pool: no decision
    assert a.should_scale_up(1, 3, 3, 500, 30.0) is None       # at max
    assert a.should_scale_down(1, 2, 2, 0, 61.0) is None       # scaled up within the cooldown
    now[0] += 100
    assert a.should_scale_down(1, 2, 2, 0, 61.0) == 1
    assert a.should_scale_down(1, 1, 1, 0, 100.0) is None      # at min
    with pytest.raises(ValueError):
        ScalingPolicy(min_replicas=0).validate()


def test_registry_transitions_and_rollback():
    from kapsl_sdk_b200.runtime.registry import ModelInfo, ModelRegistry, ModelStatus

    reg = ModelRegistry()
    events = []
    reg.add_listener(lambda *e: events.append(e[0]))
    reg.register(ModelInfo(1, "m"))
    assert reg.update_status(1, ModelStatus.STOPPING)
    assert reg.update_status(1, ModelStatus.INACTIVE)
    assert not reg.update_status(1, ModelStatus.LOADING)  # not an allowed transition
    assert reg.update_status(1, ModelStatus.STARTING)
    assert reg.rollback_status(1) == ModelStatus.INACTIVE
    reg.record_latency(1, 10)
    reg.record_latency(1, 30)
    assert reg.latency_summary(1)["p99"] == 30
    reg.register(ModelInfo(2, "m", replica_id=1, base_model_id=1))
    assert [m.id for m in reg.replicas_of(1)] == [1, 2] and reg.next_id() == 3
    assert "registered" in events and "status_changed" in events


def test_cron_interval_expression_and_skip_if_busy():
    from kapsl_sdk_b200.runtime.cron import CronExpression, CronJob, CronScheduler
    import datetime as dt

    e = CronExpression("*/15 * * * * *")
    t = dt.datetime(2026, 1, 1, 0, 0, 1)
    assert e.next_after(t).second == 15
    now = [0.0]
    s = Scheduler([Echo()], max_micro_batch=1)
    cron = CronScheduler(s, clock=lambda: now[0])
    got = []
    job = CronJob("j1", pkt(b"tick"), interval_s=5, callback=lambda jid, out: got.append(out.data))
    cron.register(job)
    now[0] = 5.0
    assert cron.tick() == 1
    now[0] = 7.0
    assert cron.tick() == 0
    assert got == [b"tick"] and job.fired == 1
    with pytest.raises(ValueError):
        cron.register(CronJob("bad", pkt(), expression="* * *"))
    busy = Scheduler([Echo(delay=0.3)], queue_size=1, max_micro_batch=1)
    c2 = CronScheduler(busy, clock=lambda: now[0])
    j2 = CronJob("j2", pkt(), interval_s=1)
    c2.register(j2)
    fut = busy.try_infer(InferenceRequest(pkt()))
    busy.try_infer(InferenceRequest(pkt())) if False else None
    now[0] = 10.0
    c2.tick()
    fut.result(timeout=5)
    assert j2.fired + j2.missed == 1
    s.shutdown()
    busy.shutdown()


def test_device_preference_and_probe():
    from kapsl_sdk_b200.hal.device import Device, DeviceBackend, DeviceInfo, GpuPreference

    gpus = [Device(0, "NVIDIA B200", DeviceBackend.CUDA, 183359, compute_capability=(10, 0), pci_bus_id="0000:1A:00.0"),
            Device(1, "NVIDIA H100", DeviceBackend.CUDA, 81559, compute_capability=(9, 0), partition_id="MIG-abc")]
    info = DeviceInfo(8, 1000, gpus)
    assert info.best_gpu().id == 0 and info.get_best_provider() == "cuda"
    assert info.select("cuda:1").id == 1
    assert info.select("0000:1a:00.0").id == 0
    assert info.select("h100").id == 1
    assert info.select("mig:MIG-abc").id == 1
    assert GpuPreference.parse("  ") is None


def test_mesh_groups_and_mock_collectives():
    from kapsl_sdk_b200.hal.mesh import DeviceMesh, DistributedOps, MeshTopology, MockComm, ReduceOp

    m = DeviceMesh(MeshTopology.mixed(tp=2, pp=2, dp=2), rank=5)
    assert m.coords() == (1, 0, 1)
    assert m.groups["tp_dp1_pp0"].ranks == [4, 5] and m.groups["pp_stage_1"].ranks == [2, 3, 6, 7]
    comms = MockComm.create_group(4)
    out = [None] * 4

    def run(c):
        ops = DistributedOps(c)
        s = ops.all_reduce_f32(np.full(4, c.rank + 1.0))
        g = ops.all_gather_f32(np.array([c.rank], np.float32))
        sc = ops.scatter_f32(np.arange(8, dtype=np.float32), root=0)
        mx = c.all_reduce(np.array([c.rank]), ReduceOp.MAX)
        c.barrier()
        out[c.rank] = (s, g, sc, mx)

    ts = [threading.Thread(target=run, args=(c,)) for c in comms]
    [t.start() for t in ts]
    [t.join() for t in ts]
    for r, (s, g, sc, mx) in enumerate(out):
        assert (s == 10).all() and list(g) == [0, 1, 2, 3] and list(sc) == [2 * r, 2 * r + 1] and mx[0] == 3


def test_mock_comm_times_out_instead_of_hanging():
    from kapsl_sdk_b200.hal.mesh import MockComm

    comms = MockComm.create_group(2)
    MockComm.TIMEOUT_S, old = 0.2, MockComm.TIMEOUT_S
    try:
        with pytest.raises(TimeoutError):
            comms[0].all_reduce(np.ones(2))  # rank 1 never joins
    finally:
        MockComm.TIMEOUT_S = old


def test_monitoring_middleware_metrics_names():
    from kapsl_sdk_b200.monitor import KapslMetrics, MonitoringMiddleware

    km = KapslMetrics()
    mw = MonitoringMiddleware(Echo(), km, model="echo")
    mw.infer(InferenceRequest(BinaryTensorPacket([2, 1], TensorDtype.UINT8, b"ab")))
    list(mw.infer_stream(InferenceRequest(pkt())))
    with pytest.raises(EngineError):
        MonitoringMiddleware(Echo(fail=True), km, model="bad").infer(InferenceRequest(pkt()))
    text = km.exposition().decode()
    for name in ("kapsl_inference_latency_seconds_bucket", "kapsl_inference_total", "kapsl_active_inferences",
                 "kapsl_batch_size", "kapsl_ttft_seconds", "kapsl_output_tokens_total"):
        assert name in text, name
    assert 'status="error"' in text
    assert mw.model_info().peak_concurrency == 1


def test_engine_pool_lru_and_health():
    from kapsl_sdk_b200.runtime.backends import EnginePool

    evicted = []

    class E(Echo):
        healthy = True

        def health_check(self):
            return self.healthy

    pool = EnginePool(capacity=2, on_evict=evicted.append)
    a, b, c = E(), E(), E()
    pool.put(1, 0, a)
    pool.put(2, 0, b)
    assert pool.get(1, 0) is a
    pool.put(3, 0, c)  # evicts (2, 0): least recently used
    assert evicted == [(2, 0)]
    a.healthy = False
    assert pool.get(1, 0) is None and (1, 0) in evicted


def test_backend_factory_requirements():
    from kapsl_sdk_b200.hal.device import Device, DeviceBackend, DeviceInfo
    from kapsl_sdk_b200.runtime.backends import BackendFactory
    from kapsl_sdk_b200.runtime.loader import Manifest

    info = DeviceInfo(8, 64000, [Device(0, "B200", DeviceBackend.CUDA, 183359, compute_capability=(10, 0))],
                      cuda_version="12.8")
    f = BackendFactory(info)
    man = Manifest.from_dict({"project_name": "m", "framework": "llm", "version": "1", "model_file": "x",
                              "hardware_requirements": {"preferred_provider": "cuda", "min_vram_mb": 200000,
                                                        "min_cuda_version": "13.0", "strategy": "tensor-parallel",
                                                        "gpu_device_ids": [0, 1]}})
    errs = f.validate_requirements(man, "cuda")
    assert len(errs) == 3
    assert f.provider_chain(man.hardware_requirements) == ["cuda", "cpu"]
    assert BackendFactory(DeviceInfo(8, 64000, [])).provider_chain(man.hardware_requirements) == ["cpu"]


def test_metrics_http_exporter():
    import urllib.request

    from kapsl_sdk_b200.monitor import KapslMetrics, serve_metrics

    m = KapslMetrics()
    m.out_tokens.labels("llm").inc(7)
    m.ttft.labels("llm").observe(0.12)
    srv = serve_metrics(m, port=0)
    try:
        port = srv.server_address[1]
        body = urllib.request.urlopen(f"http://127.0.0.1:{port}/metrics", timeout=5).read().decode()
        assert 'kapsl_output_tokens_total{model="llm"} 7.0' in body and "kapsl_ttft_seconds_bucket" in body
    finally:
        srv.shutdown()


def test_replica_with_failed_engine_is_routed_around():
    """An engine whose device step failed reports health_check() False: its
    scheduler turns unhealthy and the pool routes every request to the other
    replica, without first trying the failed one."""
    from kapsl_sdk_b200.runtime.replica_pool import PoolStrategy, ReplicaPool

    class Failed(Echo):
        failed = True

        def health_check(self):
            return False

        def infer(self, req):
            raise AssertionError("a failed replica must not be tried")

    bad, good = Scheduler([Failed()]), Scheduler([Echo()])
    pool = ReplicaPool(PoolStrategy.ROUND_ROBIN)
    pool.add_replica(0, bad)
    pool.add_replica(1, good)
    try:
        assert not bad.is_healthy() and good.is_healthy()
        assert pool.healthy_count() == 1
        for i in range(4):
            assert pool.infer(InferenceRequest(pkt(bytes([i])))).data == bytes([i])
    finally:
        for x in (bad, good):
            x.shutdown()


def test_native_work_queue_under_concurrent_producers_and_consumers():
    """The scheduler's native queue: 4 producers block on a capacity-8 queue while
    2 consumers take micro-batches; every job comes out exactly once, batches never
    exceed their size, and the depth returns to zero once the work is done."""
    import threading

    from kapsl_sdk_b200._ext import native

    q = native().WorkQueue(8)
    seen, sizes, lock = [], [], threading.Lock()

    def produce(p):
        for i in range(500):
            ok, evicted = q.put((p, i), 0, True)
            assert ok and evicted is None

    def consume():
        while True:
            batch = q.take(4, 0.001)
            if not batch:
                if q.closed:
                    return
                continue
            with lock:
                seen.extend(batch)
                sizes.append(len(batch))
            q.done(len(batch))

    cons = [threading.Thread(target=consume) for _ in range(2)]
    prods = [threading.Thread(target=produce, args=(p,)) for p in range(4)]
    [t.start() for t in cons + prods]
    [t.join(60) for t in prods]
    while q.depth():
        time.sleep(0.01)
    q.close()
    [t.join(60) for t in cons]
    assert sorted(seen) == [(p, i) for p in range(4) for i in range(500)]
    assert max(sizes) <= 4 and q.depth() == 0
    # overflow policies
    q2 = native().WorkQueue(1)
    assert q2.put("a", 0, True) == (True, None)
    assert q2.put("b", 1, True) == (False, None)      # drop newest: rejected
    assert q2.put("c", 0, False) == (False, None)     # non-blocking put on a full queue
    assert q2.put("d", 2, True) == (True, "a")        # drop oldest: "a" evicted
    assert q2.take(4, 0.0) == ["d"]


def test_device_info_helpers_follow_the_reference():
    from kapsl_sdk_b200.hal.device import Device, DeviceBackend, DeviceInfo, GpuPreference

    def dev(i, b, mem, **kw):
        return Device(i, f"dev{i}", b, mem, **kw)

    info = DeviceInfo(8, 1000, [dev(0, DeviceBackend.CPU, 1024), dev(1, DeviceBackend.CUDA, 12000),
                                dev(2, DeviceBackend.METAL, 8000)])
    assert info.best_gpu().id == 1 and [d.id for d in info.cuda_devices()] == [1]
    assert DeviceInfo(8, 1000, [dev(0, DeviceBackend.CPU, 1024)]).best_gpu() is None
    assert DeviceInfo(8, 1000, [dev(0, DeviceBackend.METAL, 9000)]).best_gpu().id == 0  # any accelerator
    assert info.get_best_provider() == "cuda"
    assert all(info.has_provider(p) for p in ("cuda", "metal", "coreml", "cpu", " CUDA "))
    assert not info.has_provider("rocm")
    assert DeviceInfo(8, 1000, [dev(0, DeviceBackend.ROCM, 9000)]).get_best_provider() == "rocm"
    parts = DeviceInfo(8, 1000, [dev(0, DeviceBackend.CPU, 1), dev(0, DeviceBackend.CUDA, 8000, partition_id="GPU-aaa"),
                                 dev(1, DeviceBackend.CUDA, 8000, partition_id="GPU-bbb")])
    assert parts.best_gpu_with_preference(GpuPreference.parse("partition:GPU-BBB")).id == 1
    assert parts.best_gpu_with_preference(GpuPreference.parse("mig:GPU-ccc")) is None
    a100 = Device(0, "NVIDIA A100 80GB PCIe", DeviceBackend.CUDA, 8000, pci_bus_id="0000:03:00.0")
    assert GpuPreference.parse("a100").matches(a100) and GpuPreference.parse("80GB").matches(a100)
    assert not GpuPreference.parse("H100").matches(a100)
    assert GpuPreference.parse("0000:03:00.0".upper()).matches(a100)
    assert not GpuPreference.parse("0000:04:00.0").matches(a100)
    assert GpuPreference.parse("cuda:0").matches(a100) and not GpuPreference.parse("cuda:2").matches(a100)
    assert GpuPreference.parse("") is None and GpuPreference.parse("  ") is None


def test_requirement_check_matches_the_reference_cases():
    """The reference factory tests' cases: host memory, VRAM and CUDA version
    minimums on the requested device, missing providers and their fallbacks,
    unknown device ids and multi-device strategies, with its error texts."""
    from kapsl_sdk_b200.hal.device import Device, DeviceBackend, DeviceInfo
    from kapsl_sdk_b200.runtime.backends import BackendFactory
    from kapsl_sdk_b200.runtime.loader import HardwareRequirements as HR

    info = DeviceInfo(8, 16 * 1024, [Device(0, "cpu", DeviceBackend.CPU, 16 * 1024),
                                     Device(1, "RTX 3080", DeviceBackend.CUDA, 10 * 1024)], cuda_version="12.0")
    check = BackendFactory.check_requirements
    assert check(HR(min_memory_mb=8 * 1024), info) is None
    assert "Insufficient memory" in check(HR(min_memory_mb=32 * 1024), info)
    assert check(HR(preferred_provider="cuda", device_id=1, min_vram_mb=8 * 1024), info) is None
    assert "insufficient VRAM" in check(HR(preferred_provider="cuda", device_id=1, min_vram_mb=12 * 1024), info)
    assert check(HR(preferred_provider="cuda", device_id=1, min_cuda_version="11.8"), info) is None
    assert "CUDA version too old" in check(HR(preferred_provider="cuda", device_id=1, min_cuda_version="12.1"), info)
    assert "Provider metal not available" in check(HR(preferred_provider="metal"), info)
    assert check(HR(preferred_provider="metal", fallback_providers=["cpu"]), info) is None
    assert "Device ID 99 not found" in check(HR(preferred_provider="cuda", device_id=99), info)
    assert check(HR(preferred_provider="cuda", min_vram_mb=9 * 1024, strategy="pool"), info) is None
    assert "No devices meet requirements" in check(HR(preferred_provider="cuda", min_vram_mb=20000, strategy="pool"),
                                                  info)
    assert check(HR(), info) is None


def test_engine_pool_warmup_skips_failures_and_reports_metrics():
    from kapsl_sdk_b200.engine_api import EngineError
    from kapsl_sdk_b200.runtime.backends import EnginePool

    class Eng:
        def __init__(self):
            self.healthy = True

        def health_check(self):
            return self.healthy

        def unload(self):
            pass

    def factory(model_id, device_id):
        if model_id == 1:
            raise EngineError.backend("warmup failed")
        return Eng()

    evicted = []
    pool = EnginePool(capacity=2, on_evict=evicted.append)
    pool.warmup([(1, 0), (2, 0)], factory)
    assert len(pool) == 1 and pool.get(2, 0) is not None and pool.get(1, 0) is None
    pool.put(3, 0, Eng())
    pool.put(4, 0, Eng())  # capacity 2: (2, 0) is least recently used
    assert evicted == [(2, 0)]
    pool.get(4, 0).healthy = False
    assert pool.get(4, 0) is None  # unhealthy: removed on get
    m = pool.pool_metrics()
    assert m["hit"] == 2 and m["failure"] == 1 and m["evictions"] == 1 and abs(m["hit_rate"] - 2 / 3) < 1e-9
