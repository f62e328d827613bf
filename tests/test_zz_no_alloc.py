"""Allocation-free C entry point of the split-KV decode attention.

Calls the exported ``kapsl_decode_attention_noalloc`` symbol of the CUDA
extension through ctypes and compares its output with the tensor API
(``ops.decode_attention``, which takes caller-allocated split scratch) and with
the plain fp32 attention oracle on two consecutive calls.  The file name sorts
last so the test also runs after the rest of the GPU suite in one process.
"""
import ctypes
import math
import random

import pytest
import torch

pytestmark = pytest.mark.gpu

HQ, HKV, D = 28, 4, 128


def _lib():
    from kapsl_sdk_b200 import _cuda

    lib = ctypes.CDLL(_cuda.__file__)
    fn = lib.kapsl_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
                   ctypes.c_void_p]
    lib.kapsl_decode_attention_noalloc_setup.restype = ctypes.c_int
    lib.kapsl_noalloc_last_error.restype = ctypes.c_char_p
    lib.kapsl_noalloc_read_and_clear_error.restype = ctypes.c_int
    lib.kapsl_noalloc_read_and_clear_error.argtypes = [ctypes.POINTER(ctypes.c_int)]
    return lib


def _fallback_err(lib) -> int:
    v = ctypes.c_int(-1)
    assert lib.kapsl_noalloc_read_and_clear_error(ctypes.byref(v)) == 0, lib.kapsl_noalloc_last_error()
    return v.value


def _case(dev, lens, seed):
    g = torch.Generator().manual_seed(seed)
    rnd = random.Random(seed)
    nb = sum((L + 15) // 16 for L in lens) + 5
    kc = torch.randn(nb, HKV, 16, D, generator=g).to(dev, torch.bfloat16)
    vc = torch.randn(nb, HKV, 16, D, generator=g).to(dev, torch.bfloat16)
    perm = list(range(nb))
    rnd.shuffle(perm)
    maxb = max((L + 15) // 16 for L in lens) + 1
    bt = torch.zeros(len(lens), maxb, dtype=torch.int32)
    p = 0
    for i, L in enumerate(lens):
        n = (L + 15) // 16
        bt[i, :n] = torch.tensor(perm[p:p + n])
        p += n
    q = torch.randn(len(lens), HQ * D, generator=g).to(dev, torch.bfloat16)
    ctx = torch.tensor(lens, dtype=torch.int32, device=dev)
    return q, kc, vc, bt.to(dev), ctx


def _oracle(q, kc, vc, bt, lens):
    """fp32 attention of each row over its gathered pages: [B, HQ, D]."""
    from kapsl_sdk_b200.ops import reference as ref

    out = []
    kcc, vcc, btc = kc.cpu(), vc.cpu(), bt.cpu()
    for i, L in enumerate(lens):
        blocks = btc[i, :(L + 15) // 16].tolist()
        k = ref.gather_paged(kcc, blocks, L)
        v = ref.gather_paged(vcc, blocks, L)
        out.append(ref.attention(q[i].view(1, HQ, D).cpu(), k, v, 1 / math.sqrt(D), L - 1)[0])
    return torch.stack(out)


def _call(lib, q, kc, vc, bt, ctx, out, nsplit, err):
    st = torch.cuda.current_stream(q.device).cuda_stream
    return lib.kapsl_decode_attention_noalloc(
        q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), kc.shape[0], bt.data_ptr(), bt.shape[1],
        ctx.data_ptr(), out.data_ptr(), out.stride(0), q.shape[0], HQ, HKV, nsplit, D ** -0.5,
        err.data_ptr() if err is not None else None, st)


def test_noalloc_matches_tensor_api():
    from kapsl_sdk_b200 import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib()
    assert lib.kapsl_decode_attention_noalloc_setup() == 0, lib.kapsl_noalloc_last_error()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    cases = [([1, 17, 300, 1025, 64, 5], 7, 0), ([2048, 33, 700], 16, 1)]
    for lens, nsplit, seed in cases:
        q, kc, vc, bt, ctx = _case(dev, lens, seed)
        want = ops.decode_attention(q, kc, vc, bt, ctx, HQ, HKV, num_splits=nsplit)
        exact = _oracle(q, kc, vc, bt, lens)
        for _ in range(2):  # two consecutive calls reuse the same static scratch
            out = torch.full_like(want, float("nan"))
            rc = _call(lib, q, kc, vc, bt, ctx, out, nsplit, err)
            assert rc == 0, lib.kapsl_noalloc_last_error()
            torch.cuda.synchronize()
            torch.testing.assert_close(out.float(), want.float(), atol=2e-2, rtol=2e-2)
            torch.testing.assert_close(out.float().cpu().view(len(lens), HQ, D), exact, atol=2e-2, rtol=2e-2)
        assert int(err.item()) == 0


def test_noalloc_rejects_oversize():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib()
    q, kc, vc, bt, ctx = _case(dev, [40, 50], 2)
    out = torch.zeros(2, HQ * D, device=dev, dtype=torch.bfloat16)
    # 2 rows * 28 heads * 64 splits is within the limit; a huge batch is not
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    assert _call(lib, q, kc, vc, bt, ctx, out, 64, err) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    torch.testing.assert_close(out.float().cpu().view(2, HQ, D), _oracle(q, kc, vc, bt, [40, 50]), atol=2e-2,
                               rtol=2e-2)
    # without an err pointer the static per-device word is used; it reads back zero and is cleared
    assert _call(lib, q, kc, vc, bt, ctx, out, 64, None) == 0
    torch.cuda.synchronize()
    assert _fallback_err(lib) == 0
    big = 100000
    rc = lib.kapsl_decode_attention_noalloc(
        q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), kc.shape[0], bt.data_ptr(), bt.shape[1],
        ctx.data_ptr(), out.data_ptr(), out.stride(0), big, HQ, HKV, 4, D ** -0.5, None,
        torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 1
    assert b"exceed the static scratch limit" in lib.kapsl_noalloc_last_error()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_second_device():
    """A call on cuda:1 after calls on cuda:0: the scratch address and the
    shared-memory attribute are per device."""
    lib = _lib()
    for idx in (0, 1):
        dev = torch.device("cuda", idx)
        with torch.cuda.device(dev):
            q, kc, vc, bt, ctx = _case(dev, [300, 17, 1025], 3)
            out = torch.full((3, HQ * D), float("nan"), device=dev, dtype=torch.bfloat16)
            err = torch.zeros(1, dtype=torch.int32, device=dev)
            assert _call(lib, q, kc, vc, bt, ctx, out, 8, err) == 0, lib.kapsl_noalloc_last_error()
            torch.cuda.synchronize(dev)
            assert int(err.item()) == 0
            torch.testing.assert_close(out.float().cpu().view(3, HQ, D), _oracle(q, kc, vc, bt, [300, 17, 1025]),
                                       atol=2e-2, rtol=2e-2)
