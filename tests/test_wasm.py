"""The in-repo WebAssembly interpreter and its WASI preview1 host, on modules
assembled here byte by byte (tests/wasm_asm.py): control flow, integer and
float semantics, traps, bulk memory, tables, then WASI stdin/stdout, the
environment, preopened directories (read-only refusals, no escapes) and a
RAG connector packaged as a `.wasm` extension."""
import json
import math
import os
import struct
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from wasm_asm import (DROP, ELSE, END, F32, F64, I32, I64, MEMORY_GROW, MEMORY_SIZE, RETURN, SELECT,  # noqa: E402
                      UNREACHABLE, Module, block, block_t, br, br_if, br_table, call, call_indirect, f64c, fc, gget,
                      gset, i32c, i64c, if_, lget, load, loop, lset, op, store, uleb)


def native():
    from kapsl_sdk_b200._ext import native as n

    return n()


def run(mod: Module, name, *args, fuel=10**8):
    return native().wasm_call(mod.build(), name, list(args), fuel)


# ------------------------------------------------------------ core semantics
def test_recursion_loops_and_branch_tables():
    m = Module()
    fib = len(m.funcs)
    m.func([I64], [I64], lget(0) + i64c(2) + op(0x53) + if_(I64) + lget(0) + ELSE +
           lget(0) + i64c(1) + op(0x7D) + call(fib) + lget(0) + i64c(2) + op(0x7D) + call(fib) + op(0x7C) + END,
           export="fib")
    m.func([I32], [I64], i64c(1) + lset(1) + block() + loop() + lget(0) + op(0x45) + br_if(1) +
           lget(1) + lget(0) + op(0xAD) + op(0x7E) + lset(1) + lget(0) + i32c(1) + op(0x6B) + lset(0) + br(0) +
           END + END + lget(1), locals_=[(1, I64)], export="fact")
    m.func([I32], [I32], block() + block() + block() + block() + lget(0) + br_table([0, 1, 2], 3) +
           END + i32c(10) + RETURN + END + i32c(20) + RETURN + END + i32c(30) + RETURN + END + i32c(99),
           export="switch")
    t2 = m.type([I32, I32], [I32])
    t0 = m.type([], [I32, I32])
    m.func([], [I32], i32c(7) + i32c(5) + block_t(t2) + op(0x6B) + END + block_t(t0) + i32c(3) + i32c(4) + END +
           op(0x6C) + op(0x6A), export="multi")
    m.func([], [I32, I64], i32c(-3) + i64c(-4), export="pair")
    m.func([I32, I32, I32], [I32], lget(0) + lget(1) + lget(2) + SELECT, export="select")
    assert run(m, "fib", 20) == [6765]
    assert run(m, "fact", 20) == [2432902008176640000]
    assert [run(m, "switch", i)[0] for i in range(6)] == [10, 20, 30, 99, 99, 99]
    assert run(m, "multi") == [2 + 12]
    assert run(m, "pair") == [-3, -4]
    assert run(m, "select", 1, 2, 1) == [1] and run(m, "select", 1, 2, 0) == [2]


def test_integer_semantics():
    m = Module()
    for name, code, t in [("div_s", 0x6D, I32), ("div_u", 0x6E, I32), ("rem_s", 0x6F, I32), ("rem_u", 0x70, I32),
                          ("shr_s", 0x75, I32), ("shr_u", 0x76, I32), ("rotl", 0x77, I32), ("rotr", 0x78, I32),
                          ("mul64", 0x7E, I64), ("div64_s", 0x7F, I64), ("shl64", 0x86, I64), ("rotl64", 0x89, I64),
                          ("lt_u", 0x49, I32)]:
        m.func([t, t], [I32 if name == "lt_u" else t], lget(0) + lget(1) + op(code), export=name)
    for name, code, t in [("clz", 0x67, I32), ("ctz", 0x68, I32), ("popcnt", 0x69, I32), ("clz64", 0x79, I64),
                          ("ext8", 0xC0, I32), ("ext16", 0xC1, I32), ("ext32_64", 0xC4, I64), ("eqz", 0x45, I32)]:
        m.func([t], [t], lget(0) + op(code), export=name)
    m.func([I64], [I32], lget(0) + op(0xA7), export="wrap")
    m.func([I32], [I64], lget(0) + op(0xAC), export="extend_s")
    m.func([I32], [I64], lget(0) + op(0xAD), export="extend_u")
    assert run(m, "div_s", -7, 2) == [-3] and run(m, "rem_s", -7, 2) == [-1]
    assert run(m, "div_u", -7, 2) == [(2**32 - 7) // 2] and run(m, "rem_u", -7, 2) == [(2**32 - 7) % 2]
    assert run(m, "rem_s", -2**31, -1) == [0]
    with pytest.raises(RuntimeError, match="integer divide by zero"):
        run(m, "div_s", 1, 0)
    with pytest.raises(RuntimeError, match="integer overflow"):
        run(m, "div_s", -2**31, -1)
    with pytest.raises(RuntimeError, match="integer overflow"):
        run(m, "div64_s", -2**63, -1)
    assert run(m, "shr_s", -16, 2) == [-4] and run(m, "shr_u", -16, 34) == [(2**32 - 16) >> 2]
    assert run(m, "rotl", 0x12345678, 8) == [0x34567812] and run(m, "rotr", 0x12345678, 8) == [0x78123456]
    assert run(m, "mul64", 2**62, 4) == [0] and run(m, "shl64", 1, 65) == [2]
    assert run(m, "rotl64", -2**63, 1) == [1]
    assert run(m, "lt_u", -1, 1) == [0]
    assert run(m, "clz", 1) == [31] and run(m, "clz", 0) == [32] and run(m, "ctz", 0) == [32]
    assert run(m, "popcnt", -1) == [32] and run(m, "clz64", 1) == [63]
    assert run(m, "ext8", 0xFF) == [-1] and run(m, "ext16", 0x8000) == [-32768] and run(m, "ext32_64", 2**31) == [-2**31]
    assert run(m, "eqz", 0) == [1] and run(m, "eqz", 5) == [0]
    assert run(m, "wrap", 2**40 + 5) == [5]
    assert run(m, "extend_s", -1) == [-1] and run(m, "extend_u", -1) == [2**32 - 1]


def test_float_semantics():
    m = Module()
    m.func([F64, F64], [F64], lget(0) + lget(1) + op(0xA4), export="min")
    m.func([F64, F64], [F64], lget(0) + lget(1) + op(0xA5), export="max")
    m.func([F64], [F64], lget(0) + op(0x9F), export="sqrt")
    m.func([F64], [F64], lget(0) + op(0x9E), export="nearest")
    m.func([F64], [F64], lget(0) + op(0x9A), export="neg")
    m.func([F64], [I32], lget(0) + op(0xAA), export="trunc_s")
    m.func([F64], [I32], lget(0) + op(0xAB), export="trunc_u")
    m.func([F64], [I32], lget(0) + fc(2), export="sat_s")
    m.func([F64], [I64], lget(0) + fc(7), export="sat_u64")
    m.func([F32, F32], [F32], lget(0) + lget(1) + op(0x92), export="add32")
    m.func([I64], [F64], lget(0) + op(0xBA), export="u64_to_f64")
    m.func([F64], [I64], lget(0) + op(0xBD), export="bits")
    m.func([F64], [F32], lget(0) + op(0xB6), export="demote")
    m.func([F64, F64], [F64], lget(0) + lget(1) + op(0xA6), export="copysign")
    assert run(m, "min", -0.0, 0.0)[0] == 0.0 and math.copysign(1, run(m, "min", 0.0, -0.0)[0]) == -1
    assert math.copysign(1, run(m, "max", -0.0, 0.0)[0]) == 1
    assert math.isnan(run(m, "min", float("nan"), 1.0)[0]) and math.isnan(run(m, "max", 1.0, float("nan"))[0])
    assert run(m, "sqrt", 2.0) == [math.sqrt(2.0)]
    assert [run(m, "nearest", x)[0] for x in (2.5, 3.5, -2.5, 0.4)] == [2.0, 4.0, -2.0, 0.0]
    assert math.copysign(1, run(m, "neg", 0.0)[0]) == -1
    assert run(m, "trunc_s", -2.9) == [-2] and run(m, "trunc_u", 4294967295.5) == [-1]
    for bad, msg in ((float("nan"), "invalid conversion"), (3e9, "integer overflow"), (-2147483649.0, "overflow")):
        with pytest.raises(RuntimeError, match=msg):
            run(m, "trunc_s", bad)
    with pytest.raises(RuntimeError, match="integer overflow"):
        run(m, "trunc_u", -1.0)
    assert run(m, "trunc_u", -0.9) == [0]
    assert run(m, "sat_s", 1e10) == [2**31 - 1] and run(m, "sat_s", -1e10) == [-2**31]
    assert run(m, "sat_s", float("nan")) == [0] and run(m, "sat_u64", -5.0) == [0] and run(m, "sat_u64", 1e30) == [-1]
    assert run(m, "add32", 0.1, 0.2) == [struct.unpack("<f", struct.pack("<f", struct.unpack("<f", struct.pack(
        "<f", 0.1))[0] + struct.unpack("<f", struct.pack("<f", 0.2))[0]))[0]]
    assert run(m, "u64_to_f64", -1) == [18446744073709551616.0]
    assert run(m, "bits", 1.0) == [0x3FF0000000000000]
    assert run(m, "demote", 1e300) == [float("inf")]
    assert run(m, "copysign", 3.0, -0.0) == [-3.0]


def test_memory_tables_globals_and_bulk_ops():
    m = Module()
    m.memory = (1, 2)
    m.datas.append((None, b"hello"))  # passive
    m.datas.append((16, b"\x01\x02\x03\x04"))  # active
    g = m.global_(I32, True, i32c(5))
    body = (i32c(8) + i32c(-1) + store(0x36) + i32c(8) + load(0x30) + i32c(8) + load(0x33) + op(0x7C) +
            i32c(1) + MEMORY_GROW + op(0xAD) + op(0x7C) +
            i32c(1) + MEMORY_GROW + op(0xAC) + op(0x7C) +
            MEMORY_SIZE + op(0xAD) + op(0x7C))
    m.func([], [I64], body, export="mem")
    m.func([], [I32], i32c(100) + i32c(0) + i32c(5) + fc(8, uleb(0), b"\x00") +
           i32c(200) + i32c(100) + i32c(5) + fc(10, b"\x00\x00") +
           i32c(300) + i32c(0x41) + i32c(3) + fc(11, b"\x00") +
           i32c(200) + load(0x28) + i32c(300) + load(0x2D) + op(0x6A), export="bulk")
    m.func([], [I32], i32c(16) + load(0x28), export="active")
    m.func([], [I32], gget(g) + i32c(1) + op(0x6A) + gset(g) + gget(g), export="inc")
    m.func([I32], [I32], lget(0) + load(0x28), export="peek")
    add = m.func([I32, I32], [I32], lget(0) + lget(1) + op(0x6A))
    mul = m.func([I32, I32], [I32], lget(0) + lget(1) + op(0x6C))
    neg = m.func([I32], [I32], i32c(0) + lget(0) + op(0x6B))
    t = m.type([I32, I32], [I32])
    m.table = 4
    m.elems.append((0, [add, mul, neg]))
    m.func([I32, I32, I32], [I32], lget(0) + lget(1) + lget(2) + call_indirect(t), export="dispatch")
    assert run(m, "mem") == [(-1 + 65535) + 1 + (-1) + 2]
    assert run(m, "bulk") == [int.from_bytes(b"hell", "little") + 0x41]
    assert run(m, "active") == [0x04030201]
    assert run(m, "inc") == [6]
    assert run(m, "dispatch", 6, 7, 0) == [13] and run(m, "dispatch", 6, 7, 1) == [42]
    with pytest.raises(RuntimeError, match="indirect call type mismatch"):
        run(m, "dispatch", 6, 7, 2)
    with pytest.raises(RuntimeError, match="uninitialized element"):
        run(m, "dispatch", 6, 7, 3)
    with pytest.raises(RuntimeError, match="undefined element"):
        run(m, "dispatch", 6, 7, 9)
    with pytest.raises(RuntimeError, match="out of bounds memory access"):
        run(m, "peek", 65533)


def test_traps_and_limits_end_the_run():
    m = Module()
    m.func([], [], UNREACHABLE, export="boom")
    m.func([], [], loop() + br(0) + END, export="spin")
    rec = len(m.funcs)
    m.func([], [], call(rec), export="recurse")
    with pytest.raises(RuntimeError, match="unreachable"):
        run(m, "boom")
    with pytest.raises(RuntimeError, match="fuel exhausted"):
        run(m, "spin", fuel=100000)
    with pytest.raises(RuntimeError, match="call stack exhausted"):
        run(m, "recurse")
    with pytest.raises(ValueError, match="not a WebAssembly module"):
        native().wasm_call(b"\x7fELF....", "x", [])
    with pytest.raises(ValueError, match="no exported function"):
        run(m, "missing")
    truncated = m.build()[:-3]
    with pytest.raises(ValueError):
        native().wasm_call(truncated, "boom", [])


# --------------------------------------------------------------------- WASI
W = "wasi_snapshot_preview1"
P4 = [I32] * 4


def echo_module() -> bytes:
    m = Module()
    rd = m.import_func(W, "fd_read", P4, [I32])
    wr = m.import_func(W, "fd_write", P4, [I32])
    m.memory = (1, None)
    m.func([], [], block() + loop() +
           i32c(0) + i32c(64) + store(0x36) + i32c(4) + i32c(1024) + store(0x36) +
           i32c(0) + i32c(0) + i32c(1) + i32c(8) + call(rd) + DROP +
           i32c(8) + load(0x28) + op(0x45) + br_if(1) +
           i32c(4) + i32c(8) + load(0x28) + store(0x36) +
           i32c(1) + i32c(0) + i32c(1) + i32c(12) + call(wr) + DROP + br(0) + END + END, export="_start")
    return m.build()


def test_wasi_stdin_stdout_env_and_exit():
    n = native()
    data = bytes(range(256)) * 20  # several 1 KiB reads
    code, out, err = n.wasm_run(echo_module(), data)
    assert code == 0 and out == data and err == b""
    code, out, _ = n.wasm_run(echo_module(), b"x" * 5000, stdout_cap=100)
    assert out == b"x" * 100  # capped
    m = Module()
    sizes = m.import_func(W, "environ_sizes_get", [I32, I32], [I32])
    get = m.import_func(W, "environ_get", [I32, I32], [I32])
    wr = m.import_func(W, "fd_write", P4, [I32])
    ex = m.import_func(W, "proc_exit", [I32], [])
    m.memory = (1, None)
    m.func([], [], i32c(0) + i32c(4) + call(sizes) + DROP + i32c(16) + i32c(1024) + call(get) + DROP +
           i32c(8) + i32c(1024) + store(0x36) + i32c(12) + i32c(4) + load(0x28) + store(0x36) +
           i32c(1) + i32c(8) + i32c(1) + i32c(2000) + call(wr) + DROP + i32c(7) + call(ex), export="_start")
    code, out, _ = n.wasm_run(m.build(), b"", [("A", "1"), ("B", "two")])
    assert code == 7 and out == b"A=1\x00B=two\x00"


def open_module(path: bytes, oflags=0, rights=2, dirfd=3) -> bytes:
    """path_open(dirfd, path) then proc_exit(errno); on success copies the file to stdout."""
    m = Module()
    po = m.import_func(W, "path_open", [I32, I32, I32, I32, I32, I64, I64, I32, I32], [I32])
    rd = m.import_func(W, "fd_read", P4, [I32])
    wr = m.import_func(W, "fd_write", P4, [I32])
    ex = m.import_func(W, "proc_exit", [I32], [])
    m.memory = (1, None)
    m.datas.append((500, path))
    m.func([], [], i32c(dirfd) + i32c(0) + i32c(500) + i32c(len(path)) + i32c(oflags) + i64c(rights) + i64c(0) +
           i32c(0) + i32c(100) + call(po) + lset(0) +
           lget(0) + if_() + lget(0) + call(ex) + END +
           i32c(0) + i32c(1024) + store(0x36) + i32c(4) + i32c(1000) + store(0x36) +
           i32c(100) + load(0x28) + i32c(0) + i32c(1) + i32c(8) + call(rd) + DROP +
           i32c(4) + i32c(8) + load(0x28) + store(0x36) +
           i32c(1) + i32c(0) + i32c(1) + i32c(12) + call(wr) + DROP, locals_=[(1, I32)], export="_start")
    return m.build()


def write_module(path: bytes, text: bytes, dirfd=3) -> bytes:
    m = Module()
    po = m.import_func(W, "path_open", [I32, I32, I32, I32, I32, I64, I64, I32, I32], [I32])
    wr = m.import_func(W, "fd_write", P4, [I32])
    ex = m.import_func(W, "proc_exit", [I32], [])
    m.memory = (1, None)
    m.datas.append((500, path))
    m.datas.append((600, text))
    m.func([], [], i32c(dirfd) + i32c(0) + i32c(500) + i32c(len(path)) + i32c(1 | 8) + i64c(64) + i64c(0) +
           i32c(0) + i32c(100) + call(po) + lset(0) + lget(0) + if_() + lget(0) + call(ex) + END +
           i32c(0) + i32c(600) + store(0x36) + i32c(4) + i32c(len(text)) + store(0x36) +
           i32c(100) + load(0x28) + i32c(0) + i32c(1) + i32c(8) + call(wr) + call(ex),
           locals_=[(1, I32)], export="_start")
    return m.build()


def test_wasi_preopened_directories(tmp_path):
    n = native()
    rw, ro = tmp_path / "rw", tmp_path / "ro"
    rw.mkdir()
    ro.mkdir()
    (rw / "in.txt").write_bytes(b"document body")
    (ro / "kb.txt").write_bytes(b"read only")
    (tmp_path / "secret.txt").write_bytes(b"outside")
    os.symlink(str(tmp_path / "secret.txt"), str(rw / "link"))
    pre = [(str(rw), "/data", False), (str(ro), "/kb", True)]

    def go(mod):
        return n.wasm_run(mod, b"", [], pre)[:2]

    assert go(open_module(b"in.txt")) == (0, b"document body")
    assert go(open_module(b"./in.txt")) == (0, b"document body")
    assert go(open_module(b"kb.txt", dirfd=4)) == (0, b"read only")
    assert go(open_module(b"missing.txt"))[0] == 44  # ENOENT
    assert go(open_module(b"../secret.txt"))[0] == 76  # ENOTCAPABLE: no escape upwards
    assert go(open_module(b"/etc/passwd"))[0] == 76
    assert go(open_module(b"link"))[0] == 32  # symlinks are not followed
    assert go(open_module(b"x.txt", dirfd=9))[0] == 8  # EBADF
    # writes: allowed under the read-write preopen, refused under the read-only one
    assert go(write_module(b"out.txt", b"written by wasm"))[0] == 0
    assert (rw / "out.txt").read_bytes() == b"written by wasm"
    assert go(write_module(b"out.txt", b"nope", dirfd=4))[0] == 76
    assert not (ro / "out.txt").exists()
    with pytest.raises(ValueError, match="preopened directory does not exist"):
        n.wasm_run(echo_module(), b"", [], [(str(tmp_path / "nope"), "/x", True)])


def test_wasi_unknown_import_and_bad_signature_are_rejected():
    m = Module()
    m.import_func("env", "host_secret", [], [I32])
    m.func([], [], b"", export="_start")
    with pytest.raises(ValueError, match="unknown import env.host_secret"):
        native().wasm_run(m.build())
    m = Module()
    m.import_func(W, "fd_write", [I32], [I32])
    m.func([], [], b"", export="_start")
    with pytest.raises(ValueError, match="wrong signature"):
        native().wasm_run(m.build())
    m = Module()  # a preview1 call that is not implemented answers ENOSYS
    sock = m.import_func(W, "sock_accept", [I32, I32, I32], [I32])
    ex = m.import_func(W, "proc_exit", [I32], [])
    m.func([], [], i32c(0) + i32c(0) + i32c(0) + call(sock) + call(ex), export="_start")
    assert native().wasm_run(m.build())[0] == 52


# ----------------------------------------------------------- RAG connector
def connector_module(reply: bytes) -> bytes:
    """Drains stdin, then prints `reply` (one JSON line)."""
    m = Module()
    rd = m.import_func(W, "fd_read", P4, [I32])
    wr = m.import_func(W, "fd_write", P4, [I32])
    m.memory = (1, None)
    m.datas.append((4096, reply))
    m.func([], [], block() + loop() +
           i32c(0) + i32c(64) + store(0x36) + i32c(4) + i32c(1024) + store(0x36) +
           i32c(0) + i32c(0) + i32c(1) + i32c(8) + call(rd) + DROP +
           i32c(8) + load(0x28) + op(0x45) + br_if(1) + br(0) + END + END +
           i32c(16) + i32c(4096) + store(0x36) + i32c(20) + i32c(len(reply)) + store(0x36) +
           i32c(1) + i32c(16) + i32c(1) + i32c(24) + call(wr) + DROP, export="_start")
    return m.build()


def test_wasm_connector_extension(tmp_path):
    from kapsl_sdk_b200 import rag

    reply = json.dumps({"id": "w", "status": "Ok", "result": {"type": "Health", "value": "wasm-ok"}}).encode() + b"\n"
    src = tmp_path / "src"
    src.mkdir()
    (src / "connector.wasm").write_bytes(connector_module(reply))
    (src / "manifest.json").write_text(json.dumps({
        "id": "wdocs", "name": "Wasm docs", "version": "0.1.0", "runtime": "wasm", "capabilities": ["sync"],
        "auth": ["none"], "permissions": [], "entrypoint": "connector.wasm"}))
    reg = rag.ExtensionRegistry(str(tmp_path / "ext"))
    reg.install_from_dir(str(src))
    mgr = rag.ExtensionManager(reg, str(tmp_path / "cfg"))
    data = tmp_path / "data"
    data.mkdir()
    mgr.set_workspace_config("ws", "wdocs", {"wasi": {"env": {"TOKEN": "t"},
                                                      "preopen_dirs": [{"host_path": str(data), "guest_path": "/data",
                                                                        "read_only": True}]}})
    client = mgr.launch_connector("ws", "wdocs")
    assert client.health() == "wasm-ok"
    assert client.runtime.env == [("TOKEN", "t")] and client.runtime.preopens == [(str(data), "/data", True)]
    with pytest.raises(ValueError, match="guest path must be absolute"):
        rag.runtime.WasmRuntime(str(src / "connector.wasm"), preopens=[(str(data), "data", True)])
    with pytest.raises(ValueError, match="NUL"):
        rag.runtime.WasmRuntime(str(src / "connector.wasm"), env={"K": "a\0b"})
