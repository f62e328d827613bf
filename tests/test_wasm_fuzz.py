"""Mutation fuzzing of the in-repo WebAssembly loader and interpreter, which run
untrusted connector modules: thousands of byte-level mutations (flips, inserts,
deletes, truncations, inflated LEB128 lengths) of valid modules must each end in
a clean rejection (ValueError), a trap (RuntimeError) or a result, never a crash
of the process.  The mutations run in a child process so that a crash fails the
test with the mutation that caused it instead of taking pytest down."""
import os
import subprocess
import sys
import textwrap

CHILD = textwrap.dedent(r'''
    import os, random, sys
    sys.path.insert(0, os.environ["TESTS_DIR"])
    from wasm_asm import (DROP, END, I32, I64, MEMORY_GROW, Module, block, br, br_if, br_table, call,
                          call_indirect, gget, gset, i32c, i64c, if_, lget, load, loop, lset, op, store)
    from kapsl_sdk_b200._ext import native
    n = native()

    def mods():
        out = []
        m = Module()
        m.memory = (1, 2)
        m.func([I32, I32], [I32], lget(0) + lget(1) + op(0x6A), export="add")
        m.func([I32], [I32], block() + loop() + lget(0) + op(0x45) + br_if(1) + lget(0) + i32c(1) + op(0x6B) +
               lset(0) + br(0) + END + END + lget(0), export="count")
        m.func([I32], [I32], lget(0) + load(0x28) + i32c(3) + MEMORY_GROW + op(0x6A), export="mem")
        out.append(m.build())
        m2 = Module()
        f = m2.func([I64], [I64], lget(0) + i64c(7) + op(0x7E), export="mul")
        m2.func([I32], [I32], block() + block() + lget(0) + br_table([0, 1], 1) + END + i32c(5) + op(0x1A) +
                END + i32c(9), export="tbl")
        out.append(m2.build())
        return out

    rng = random.Random(int(sys.argv[1]))
    calls = [("add", [1, 2]), ("count", [5]), ("mem", [0]), ("mul", [3]), ("tbl", [1])]
    base = mods()
    for i in range(int(sys.argv[2])):
        b = bytearray(rng.choice(base))
        for _ in range(rng.randint(1, 4)):
            k = rng.random()
            pos = rng.randrange(len(b))
            if k < 0.45:
                b[pos] ^= 1 << rng.randrange(8)
            elif k < 0.6:
                b.insert(pos, rng.randrange(256))
            elif k < 0.75 and len(b) > 9:
                del b[pos]
            elif k < 0.85:
                b = b[:max(8, pos)]
            else:
                b[pos] = rng.choice([0x7F, 0xFF, 0x80, 0x00])
        name, args = rng.choice(calls)
        sys.stdout.write(f"{i}\n")
        sys.stdout.flush()
        try:
            n.wasm_call(bytes(b), name, args, 200000)
        except (ValueError, RuntimeError, TypeError, OverflowError):
            pass
        try:
            n.wasm_run(bytes(b), fuel=200000, timeout_s=2.0)
        except (ValueError, RuntimeError):
            pass
    print("done")
''')


def test_mutated_modules_never_crash_the_process():
    env = dict(os.environ, TESTS_DIR=os.path.dirname(os.path.abspath(__file__)))
    for seed in (1, 2):
        p = subprocess.run([sys.executable, "-c", CHILD, str(seed), "1500"], capture_output=True, text=True,
                           timeout=600, env=env, cwd=os.path.dirname(env["TESTS_DIR"]))
        last = p.stdout.strip().splitlines()[-1] if p.stdout.strip() else "none"
        assert p.returncode == 0 and last == "done", \
            f"seed {seed}: child ended with {p.returncode} after mutation {last}: {p.stderr[-2000:]}"
