"""Fuzzing of native code that reads untrusted bytes, each run in a child process so
that a crash fails the test with the input that caused it: the HNSW index loader
(truncated and mutated saved indexes load into an index that answers searches, or
raise), the shared-memory server (garbage requests from a client that shares
the region get error responses and the server keeps serving) and the socket
server's frame reader."""
import os
import subprocess
import sys
import textwrap

CHILD = textwrap.dedent(r'''
    import os, random, sys, tempfile
    import numpy as np
    from kapsl_sdk_b200._ext import native
    rg = native().rag
    d = tempfile.mkdtemp()
    h = rg.Hnsw(8, 4, 16)
    h.add(np.random.default_rng(0).standard_normal((60, 8)).astype(np.float32), 1)
    src = os.path.join(d, "i.bin")
    h.save(src)
    good = open(src, "rb").read()
    rng = random.Random(int(sys.argv[1]))
    path = os.path.join(d, "m.bin")
    for i in range(int(sys.argv[2])):
        b = bytearray(good)
        if i % 4 == 0:
            b = b[:rng.randrange(len(b))]
        else:
            for _ in range(rng.randint(1, 6)):
                b[rng.randrange(len(b))] = rng.randrange(256)
        open(path, "wb").write(bytes(b))
        sys.stdout.write(f"{i}\n")
        sys.stdout.flush()
        try:
            g = rg.Hnsw.load(path)
            g.search(np.ones(8, np.float32), 5)
        except (RuntimeError, ValueError):
            pass
    print("done")
''')


def test_corrupted_index_files_never_crash_the_process():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for seed in (1, 2):
        p = subprocess.run([sys.executable, "-c", CHILD, str(seed), "1500"], capture_output=True, text=True,
                           timeout=600, cwd=root)
        last = p.stdout.strip().splitlines()[-1] if p.stdout.strip() else "none"
        assert p.returncode == 0 and last == "done", \
            f"seed {seed}: child ended with {p.returncode} after mutation {last}: {p.stderr[-2000:]}"


SHM_CHILD = textwrap.dedent(r'''
    import random, struct, sys, time, uuid
    from kapsl_sdk_b200._ext import native
    from kapsl_sdk_b200.server.dispatch import Dispatcher

    class Echo:
        def infer(self, request, priority="throughput"):
            return request.input

    nat = native()
    name = f"kapsl-fuzz-{uuid.uuid4().hex[:8]}"
    srv = nat.ShmServer(Dispatcher(lambda i: Echo()), name, 16 << 20, 1)
    srv.start()
    region = nat.ShmRegion.open(name)
    pool = region.header()["tensor_pool_offset"]
    rng = random.Random(int(sys.argv[1]))
    junk = bytes(rng.randrange(256) for _ in range(1 << 16))
    region.write_tensor(pool, [len(junk)], "uint8", junk)  # a pool full of random bytes to point into

    def drain(wait_s, until=None):
        got, t0 = [], time.time()
        while time.time() - t0 < wait_s and not (until is not None and any(r[0] == until for r in got)):
            r = region.pop_response()
            if r is None:
                time.sleep(0.0005)
                continue
            got.append(r)
            if r[1] == 0:  # read results and error messages, as a client does, so their slots free up
                region.mark_result_read(r[2])
            elif r[4] > 0:
                region.read_error(r[4])
                region.mark_result_read(r[4])
        return got

    sizes = [0, 1, 7, 80, 4096, 1 << 20, 1 << 40, (1 << 64) - 1]
    sent = 0
    for i in range(int(sys.argv[2])):
        off = rng.choice([pool + rng.randrange(1 << 16), rng.randrange(1 << 25), (1 << 64) - 1 - rng.randrange(64),
                          pool + rng.randrange(64)])
        size = rng.choice(sizes + [rng.randrange(1 << 17)])
        if region.push_request(i + 1, rng.randrange(4), rng.randrange(256), off, size):
            sent += 1
        if i % 64 == 63:
            drain(0.01)
        sys.stdout.write(f"{i}\n")
        sys.stdout.flush()
    drain(0.5)
    # the server still serves a well-formed request
    payload = struct.pack("<4i", 1, 2, 3, 4)
    region.write_tensor(pool + (1 << 20), [4], "int32", payload)
    assert region.push_request(10 ** 9, 0, 0, pool + (1 << 20), 96)
    ok = [r for r in drain(30.0, until=10 ** 9) if r[0] == 10 ** 9]  # generous: the host may be loaded
    assert ok and ok[0][1] == 0 and region.read_tensor(ok[0][2])[2] == payload, ok
    srv.stop()
    print("done")
''')


def test_garbage_shared_memory_requests_never_crash_the_server():
    """Requests whose tensor offsets and sizes point at random bytes, past the
    region or at absurd lengths get error responses; the server keeps running and
    answers a well-formed request afterwards."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for seed in (1, 2):
        p = subprocess.run([sys.executable, "-c", SHM_CHILD, str(seed), "1500"], capture_output=True, text=True,
                           timeout=600, cwd=root)
        last = p.stdout.strip().splitlines()[-1] if p.stdout.strip() else "none"
        assert p.returncode == 0 and last == "done", \
            f"seed {seed}: child ended with {p.returncode} after request {last}: {p.stderr[-2000:]}"


SOCK_CHILD = textwrap.dedent(r'''
    import os, random, resource, socket, struct, sys, tempfile, time
    from kapsl_sdk_b200.engine_api import EngineError
    from kapsl_sdk_b200.server import KapslServer
    from kapsl_sdk_b200.server import wire as pyw

    class Echo:
        def infer(self, request, priority="throughput"):
            return request.input

        def infer_stream(self, request):
            def gen():
                for b in request.input.data[:4]:
                    yield type(request.input)(shape=[1], dtype=request.input.dtype, data=bytes([b]))
            return gen()

    sock = os.path.join(tempfile.mkdtemp(), "k.sock")
    srv = KapslServer(models={0: Echo()}).listen_unix(sock).start()
    rng = random.Random(int(sys.argv[1]))
    good = pyw.encode_request(([4], "uint8", b"abcd"))
    rss0 = resource.getrusage(resource.RUSAGE_SELF).ru_maxrss
    for i in range(int(sys.argv[2])):
        s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        s.settimeout(0.2)
        s.connect(sock)
        try:
            for _ in range(rng.randint(1, 3)):
                k = rng.random()
                body = bytearray(good)
                if k < 0.4:
                    for _ in range(rng.randint(1, 4)):
                        body[rng.randrange(len(body))] = rng.randrange(256)
                elif k < 0.6:
                    body = body[:rng.randrange(len(body))]
                elif k < 0.75:
                    body = bytearray(rng.randrange(256) for _ in range(rng.randrange(64)))
                op = rng.choice([1, 2, 3, 4, 0, 7, 0xFFFFFFFF])
                size = len(body) if rng.random() < 0.85 else rng.choice([len(body) + 5, 1 << 30, (1 << 31) + 1])
                s.sendall(struct.pack("<III", rng.randrange(3), op, size) + bytes(body))
                if size != len(body):
                    break  # the server waits for bytes that never come: hang up
                try:
                    s.recv(1 << 16)
                except OSError:
                    pass
        except OSError:
            pass
        finally:
            s.close()
        sys.stdout.write(f"{i}\n")
        sys.stdout.flush()
    grown_mb = (resource.getrusage(resource.RUSAGE_SELF).ru_maxrss - rss0) / 1024
    from kapsl_sdk import KapslClient
    assert KapslClient(sock).infer(0, [4], "uint8", b"wxyz") == b"wxyz"
    assert grown_mb < 512, grown_mb  # declared 1-2 GiB payloads were never allocated
    srv.stop()
    print("done")
''')


def test_malformed_socket_frames_never_crash_the_server():
    """Mutated, truncated and random request frames, unknown ops and headers that
    declare up to 2 GiB of payload get errors or a closed connection; the server
    keeps serving and never allocates a payload that did not arrive."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for seed in (1, 2):
        p = subprocess.run([sys.executable, "-c", SOCK_CHILD, str(seed), "400"], capture_output=True, text=True,
                           timeout=600, cwd=root)
        last = p.stdout.strip().splitlines()[-1] if p.stdout.strip() else "none"
        assert p.returncode == 0 and last == "done", \
            f"seed {seed}: child ended with {p.returncode} after connection {last}: {p.stderr[-2000:]}"
