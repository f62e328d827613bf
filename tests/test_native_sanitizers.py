"""The C++ runtime pieces that run without Python (SHM region and rings,
allocators, lease words, block allocator, bincode codec, CPU kernel pool,
WebAssembly decoder and interpreter with randomly corrupted modules)
built as one standalone program under ThreadSanitizer and under
AddressSanitizer + UndefinedBehaviorSanitizer, run here on the CPU."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "csrc", "native")
FILES = ["selftest.cpp", "shm.cpp", "wire.cpp", "block_alloc.cpp", "cpu_kernels.cpp", "wasm.cpp", "text_index.cpp", "hnsw.cpp"]


def _build(tmp_path, flags):
    exe = str(tmp_path / "selftest")
    cmd = ["g++", "-std=c++17", "-O1", "-g", *flags, *[os.path.join(SRC, f) for f in FILES], "-I", SRC, "-pthread",
           "-lrt", "-fopenmp-simd", "-mavx2", "-mfma", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    if r.returncode != 0 and "sanitize" in r.stderr:
        pytest.skip("sanitizer runtime not available: " + r.stderr[-300:])
    assert r.returncode == 0, r.stderr[-3000:]
    return exe


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_threadsanitizer(tmp_path):
    exe = _build(tmp_path, ["-fsanitize=thread"])
    env = dict(os.environ, TSAN_OPTIONS=f"suppressions={os.path.join(SRC, 'tsan.supp')} halt_on_error=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0 and "selftest ok" in r.stdout, (r.stdout + r.stderr)[-4000:]
    assert "ThreadSanitizer" not in r.stderr, r.stderr[-4000:]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_address_and_undefined_sanitizers(tmp_path):
    exe = _build(tmp_path, ["-fsanitize=address,undefined", "-fno-omit-frame-pointer"])
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1", UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0 and "selftest ok" in r.stdout, (r.stdout + r.stderr)[-4000:]
    assert "runtime error" not in r.stderr and "AddressSanitizer" not in r.stderr, r.stderr[-4000:]
