"""Corrupted-file fuzzing of the native HNSW index loader (a saved vector index is
read back from disk): truncations and byte mutations of a saved index must load
into an index that answers searches, or raise, never crash the process.  Runs in
a child process so that a crash fails the test with the mutation that caused it."""
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
