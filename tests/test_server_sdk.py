"""The C++ servers driven by the C++ client SDK over a Unix socket, TCP,
shared memory and the hybrid path (no GPU)."""
import os
import struct
import tempfile
import threading
import time
import uuid

import pytest

from kapsl_sdk_b200.engine_api import BinaryTensorPacket, EngineError, TensorDtype


class EchoTarget:
    """Echo model: output = input; streams the input bytes one by one."""

    def __init__(self, fail_after=None, fail_start=False):
        self.fail_after = fail_after
        self.fail_start = fail_start
        self.calls = 0

    def infer(self, request, priority="throughput"):
        self.calls += 1
        if request.input.data == b"boom":
            raise EngineError.inference("boom requested")
        return request.input

    def infer_stream(self, request):
        if self.fail_start:
            raise EngineError.overloaded("queue full")
        data = request.input.data

        def gen():
            for i, b in enumerate(data):
                if self.fail_after is not None and i == self.fail_after:
                    raise EngineError.inference("mid-stream failure")
                yield BinaryTensorPacket([1, 1], TensorDtype.UTF8, bytes([b]))

        return gen()


@pytest.fixture
def sock_path():
    d = tempfile.mkdtemp(prefix="kapsl-")
    yield os.path.join(d, "k.sock")


def start_server(targets, sock=None, tcp=False, token=None, shm=None):
    from kapsl_sdk_b200.server import KapslServer

    srv = KapslServer(models=targets, api_token=token)
    if sock:
        srv.listen_unix(sock)
    if tcp:
        srv.listen_tcp("127.0.0.1", 0)
    if shm:
        srv.serve_shm(shm, size=64 << 20, workers=2)
    return srv.start()


def test_unix_infer_tensor_and_stream(sock_path):
    from kapsl_sdk import KapslClient

    srv = start_server({0: EchoTarget(), 3: EchoTarget()}, sock=sock_path)
    try:
        c = KapslClient(sock_path)
        assert c.protocol() == "socket" and c.endpoint() == f"unix://{sock_path}"
        data = struct.pack("<4f", 1, 2, 3, 4)
        assert c.infer(0, [2, 2], "float32", data) == data
        out, shape, dt = c.infer_tensor(3, [4], "fp32", data)
        assert (out, shape, dt) == (data, [4], "float32")
        chunks = list(c.infer_stream(0, [1, 3], "string", b"abc"))
        assert chunks == [b"a", b"b", b"c"]
        with pytest.raises(RuntimeError, match="Model 9 not found"):
            c.infer(9, [1], "uint8", b"x")
        with pytest.raises(RuntimeError, match="Inference error: boom requested"):
            c.infer(0, [4], "uint8", b"boom")
        with pytest.raises(ValueError):
            c.infer(0, [1], "bfloat99", b"x")
        # the pooled connection stays usable after server-side errors
        assert c.infer(0, [1], "uint8", b"z") == b"z"
    finally:
        srv.stop()


def test_stream_error_ordering(sock_path):
    from kapsl_sdk import KapslClient

    srv = start_server({0: EchoTarget(fail_after=2), 1: EchoTarget(fail_start=True)}, sock=sock_path)
    try:
        c = KapslClient(socket_path=sock_path)
        it = c.infer_stream(0, [1, 4], "string", b"wxyz")
        assert next(it) == b"w" and next(it) == b"x"
        with pytest.raises(RuntimeError, match="mid-stream failure"):
            next(it)
        with pytest.raises(StopIteration):  # ERR is followed by END
            next(it)
        it = c.infer_stream(1, [1, 1], "string", b"q")
        with pytest.raises(RuntimeError, match="System overloaded: queue full"):
            next(it)
    finally:
        srv.stop()


def test_tcp_auth(sock_path):
    from kapsl_sdk import KapslClient

    srv = start_server({0: EchoTarget()}, tcp=True, token="sekret")
    try:
        port = srv.tcp_port
        ok = KapslClient(protocol="tcp", host="127.0.0.1", port=port, api_token="sekret")
        assert ok.protocol() == "tcp" and ok.endpoint() == f"tcp://127.0.0.1:{port}"
        assert ok.infer(0, [1], "uint8", b"k") == b"k"
        assert list(ok.infer_stream(0, [1, 2], "string", b"hi")) == [b"h", b"i"]
        bad = KapslClient(f"tcp://127.0.0.1:{port}", api_token="wrong")
        with pytest.raises(RuntimeError, match="^Unauthorized$"):
            bad.infer(0, [1], "uint8", b"k")
        none = KapslClient(f"tcp://127.0.0.1:{port}")
        with pytest.raises(RuntimeError, match="Unauthorized"):
            none.infer(0, [1], "uint8", b"k")
        with pytest.raises(RuntimeError, match="Unauthorized"):
            next(none.infer_stream(0, [1, 1], "string", b"k"))
    finally:
        srv.stop()


def test_endpoint_resolution_errors():
    from kapsl_sdk import KapslClient

    assert KapslClient().endpoint() == "unix:///tmp/kapsl.sock"
    assert KapslClient(port=9100).endpoint() == "tcp://127.0.0.1:9100"
    assert KapslClient(protocol="tcp").endpoint() == "tcp://127.0.0.1:9096"
    for kw in ({"endpoint": "tcp://"}, {"protocol": "carrier-pigeon"}, {"protocol": "tcp", "socket_path": "/x"},
               {"protocol": "socket", "host": "h"}, {"protocol": "pipe"}, {"pipe_name": "p"},
               {"protocol": "tcp", "endpoint": "unix:///x"}):
        with pytest.raises(ValueError):
            KapslClient(**kw)
    c = KapslClient("/nonexistent/kapsl.sock")
    with pytest.raises(ConnectionError):
        c.infer(0, [1], "uint8", b"x")


def test_live_socket_is_refused_and_stale_is_replaced(sock_path):
    srv = start_server({0: EchoTarget()}, sock=sock_path)
    try:
        with pytest.raises(RuntimeError, match="in use"):
            start_server({0: EchoTarget()}, sock=sock_path)
    finally:
        srv.stop()
    open(sock_path, "w").close()  # stale file
    srv2 = start_server({0: EchoTarget()}, sock=sock_path)
    srv2.stop()


def test_retry_on_stale_pooled_connection(sock_path):
    from kapsl_sdk import KapslClient

    srv = start_server({0: EchoTarget()}, sock=sock_path)
    c = KapslClient(sock_path)
    assert c.infer(0, [1], "uint8", b"a") == b"a"
    srv.stop()
    srv = start_server({0: EchoTarget()}, sock=sock_path)
    try:
        assert c.infer(0, [1], "uint8", b"b") == b"b"  # pooled fd is dead: one retry on a fresh one
    finally:
        srv.stop()


def test_shm_and_hybrid(sock_path):
    from kapsl_sdk import KapslHybridClient, KapslShmClient

    name = f"kapsl-test-{uuid.uuid4().hex[:8]}"
    tgt = EchoTarget()
    srv = start_server({0: tgt}, sock=sock_path, shm=name)
    try:
        c = KapslShmClient(name)
        data = struct.pack("<6i", *range(6))
        assert c.infer([2, 3], "int32", data) == data
        with pytest.raises(RuntimeError, match="boom requested"):
            c.infer([4], "uint8", b"boom")
        h = KapslHybridClient(name, sock_path)
        assert h.infer([3], "float32", struct.pack("<3f", 1, 2, 3)) == struct.pack("<3f", 1, 2, 3)
        # concurrent SHM clients do not lose each other's responses
        errs = []

        def worker(i):
            try:
                cc = KapslShmClient(name)
                for j in range(20):
                    payload = struct.pack("<2i", i, j)
                    assert cc.infer([2], "int32", payload) == payload
            except Exception as e:  # pragma: no cover - reported below
                errs.append(e)

        ts = [threading.Thread(target=worker, args=(i,)) for i in range(4)]
        [t.start() for t in ts]
        [t.join() for t in ts]
        assert not errs, errs
        assert srv.shm.requests_served >= 82
    finally:
        srv.stop()


def test_shm_rejects_out_of_bounds_offsets():
    from kapsl_sdk_b200._ext import native

    nat = native()
    name = f"kapsl-oob-{uuid.uuid4().hex[:8]}"
    srv = nat.ShmServer(__import__("kapsl_sdk_b200.server.dispatch", fromlist=["x"]).Dispatcher(
        lambda i: EchoTarget()), name, 16 << 20, 1)
    srv.start()
    try:
        region = nat.ShmRegion.open(name)
        assert region.header()["magic"] == 0x41494D4F
        assert region.push_request(1, 0, 0, (1 << 40), 100)
        for _ in range(500):
            r = region.pop_response()
            if r is not None:
                break
            time.sleep(0.01)
        rid, status, off, size, err_off = r
        assert rid == 1 and status == 1 and err_off > 0
        assert "outside" in region.read_error(err_off)
    finally:
        srv.stop()


def test_shm_unread_results_are_not_overwritten():
    """More responses than result slots while no client reads: every result the
    server did write keeps its own bytes (an unread slot is never taken over; the
    surplus requests get errors), and marking results read frees their slots."""
    from kapsl_sdk_b200._ext import native

    nat = native()
    name = f"kapsl-guard-{uuid.uuid4().hex[:8]}"
    srv = nat.ShmServer(__import__("kapsl_sdk_b200.server.dispatch", fromlist=["x"]).Dispatcher(
        lambda i: EchoTarget()), name, 16 << 20, 1)
    srv.start()
    try:
        region = nat.ShmRegion.open(name)
        base = region.header()["tensor_pool_offset"]
        slots = sum(int(c.split("x")[1]) for c in srv.pool_layout().split(": ")[1].split(","))
        n = slots + 6

        def send(i):
            payload = struct.pack("<4i", i, 2 * i, 3 * i, 4 * i)
            region.write_tensor(base + i * 4096, [4], "int32", payload)
            assert region.push_request(i + 1, 0, 0, base + i * 4096, 80 + 16)
            return payload

        payloads = {}
        got = {}
        for i in range(n):
            payloads[i + 1] = send(i)
            t0 = time.time()
            while i + 1 not in got and time.time() - t0 < 20:  # one at a time, in order
                r = region.pop_response()
                if r is None:
                    time.sleep(0.001)
                    continue
                got[r[0]] = r
        assert len(got) == n
        ok = {rid: r for rid, r in got.items() if r[1] == 0}
        assert len(ok) == slots and sorted(ok) == list(range(1, slots + 1))
        assert all(got[rid][1] != 0 for rid in range(slots + 1, n + 1))  # pool exhausted, nothing overwritten
        for rid, r in ok.items():
            assert region.read_tensor(r[2])[2] == payloads[rid]
            region.mark_result_read(r[2])
        payloads[n + 1] = send(n)
        t0 = time.time()
        r = None
        while r is None and time.time() - t0 < 20:
            r = region.pop_response()
            time.sleep(0.001)
        assert r is not None and r[0] == n + 1 and r[1] == 0
        assert region.read_tensor(r[2])[2] == payloads[n + 1]
    finally:
        srv.stop()


def test_model_pools_allocator():
    """Per-model sub-pools with a shared overflow pool: model pool first, spill
    to the shared pool, unknown ids to the shared pool, release by offset range."""
    from kapsl_sdk_b200._ext import native

    P = native().ModelPools
    MiB = 1 << 20
    plan = dict(P.plan(100 * MiB, [(7, 1), (3, 3)]))
    assert set(plan) == {3, 7}
    assert plan[3] == 3 * (90 * MiB) // 4 and plan[3] + plan[7] == 90 * MiB  # 10% stays shared
    # model 0's slice (under 64 KiB) is dropped and the last model takes the rest
    assert P.plan(1 << 20, [(0, 1), (1, 1000)]) == [(1, (1 << 20) - (1 << 20) // 10)]

    pools = P(4096, 10 * MiB, [(0, 2 * MiB, [MiB], [1]), (1, 3 * MiB, [MiB], [1])], ttl_s=60.0)
    b0, e0 = pools.range(0)
    b1, e1 = pools.range(1)
    bs, es = pools.range()
    assert (b0, e0, b1, e1, es) == (4096, 4096 + 2 * MiB, e0, e0 + 3 * MiB, 4096 + 10 * MiB) and bs == e1
    got0 = [pools.try_allocate(0, MiB) for _ in range(2)]
    assert all(b0 <= o < e0 for o in got0)
    spill = pools.try_allocate(0, MiB)  # model 0's pool is full -> shared pool
    assert bs <= spill < es
    other = pools.try_allocate(42, 1000)  # no pool of its own
    assert bs <= other < es
    assert pools.usage(0)[0] == 2 and pools.usage(1)[0] == 0 and pools.usage()[0] == 2
    assert pools.total_usage()[0] == 4
    assert pools.try_allocate(1, 8 * MiB) is None  # larger than every slot of both pools
    assert pools.release(got0[0]) and pools.usage(0)[0] == 1
    assert pools.try_allocate(0, MiB) == got0[0]
    assert pools.release(spill) and not pools.release(es + 10)
    assert "model 0" in pools.layout_summary() and "shared" in pools.layout_summary()


def test_shm_server_per_model_pools():
    from kapsl_sdk import KapslShmClient

    name = f"kapsl-pm-{uuid.uuid4().hex[:8]}"
    a, b = EchoTarget(), EchoTarget()
    b.peak_concurrency = 3
    from kapsl_sdk_b200.server import KapslServer

    srv = KapslServer(models={0: a, 1: b}).serve_shm(name, size=64 << 20, workers=2).start()
    try:
        layout = srv.shm.pool_layout()
        assert "model 0" in layout and "model 1" in layout and "shared" in layout
        c = KapslShmClient(name)  # requests model 0
        for i in range(3):
            assert c.infer([1], "int32", struct.pack("<i", i)) == struct.pack("<i", i)
        assert srv.shm.pool_usage(0)[0] == 3 and srv.shm.pool_usage(1)[0] == 0
        assert srv.shm.pool_in_use == 3
    finally:
        srv.stop()
