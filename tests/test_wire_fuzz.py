"""Property-based checks of the C++ wire codec that parses untrusted client bytes:
random valid requests and packets round-trip and equal the pure-Python encoder's
bytes; truncated, bit-flipped and random inputs never crash the decoder (they
decode or raise ValueError / RuntimeError), and declared lengths beyond the
buffer are refused without allocating them."""
import struct

import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402

from kapsl_sdk_b200.server import wire as pyw  # noqa: E402


@pytest.fixture(scope="module")
def nat():
    from kapsl_sdk_b200._ext import native

    return native()


DTYPES = {"float32": 4, "float64": 8, "float16": 2, "int32": 4, "int64": 8, "uint8": 1}
shape_st = st.lists(st.integers(1, 5), min_size=1, max_size=4)


@st.composite
def packets(draw):
    shape = draw(shape_st)
    dtype = draw(st.sampled_from(sorted(DTYPES)))
    n = 1
    for d in shape:
        n *= d
    return shape, dtype, draw(st.binary(min_size=n * DTYPES[dtype], max_size=n * DTYPES[dtype]))


text = st.text(alphabet=st.characters(codec="utf-8", exclude_categories=("Cs",)), max_size=12)
metadata_st = st.fixed_dictionaries({}, optional={
    "request_id": text, "timeout_ms": st.integers(0, 2 ** 40), "priority": st.integers(0, 255),
    "force_cpu": st.booleans(), "model_version": text, "auth_token": text,
    "max_new_tokens": st.integers(0, 2 ** 31 - 1),
    "temperature": st.floats(0, 4, width=32), "top_p": st.floats(0, 1, width=32), "top_k": st.integers(0, 2 ** 31 - 1),
    "repetition_penalty": st.floats(0.5, 2, width=32), "seed": st.integers(0, 2 ** 63 - 1),
    "stop_token_ids": st.lists(st.integers(0, 2 ** 31 - 1), max_size=4)})


@settings(max_examples=200, deadline=None)
@given(p=packets(), extra=st.lists(st.tuples(text, packets()), max_size=2), sid=st.one_of(st.none(), text),
       md=metadata_st)
def test_requests_roundtrip_and_match_python(nat, p, extra, sid, md):
    b_c = nat.encode_request({"input": p, "additional_inputs": extra, "session_id": sid, "metadata": md})
    assert b_c == pyw.encode_request(p, extra, sid, md)
    d = nat.decode_request(b_c)
    assert d["input"] == tuple(p) and d["session_id"] == sid
    assert [(n, tuple(t)) for n, t in d["additional_inputs"]] == [(n, tuple(t)) for n, t in extra]
    for k, v in md.items():
        assert d["metadata"][k] == (pytest.approx(v) if isinstance(v, float) else v)


def _decode_safely(fn, b):
    try:
        fn(b)
    except (ValueError, RuntimeError, UnicodeDecodeError):
        pass


@settings(max_examples=300, deadline=None)
@given(p=packets(), md=metadata_st, cut=st.integers(0, 10 ** 6), flips=st.lists(st.integers(0, 10 ** 6), max_size=4))
def test_truncated_and_corrupted_requests_never_crash(nat, p, md, cut, flips):
    b = bytearray(nat.encode_request({"input": p, "metadata": md}))
    for f in flips:
        b[f % len(b)] ^= 1 << (f % 8)
    _decode_safely(nat.decode_request, bytes(b))
    _decode_safely(nat.decode_request, bytes(b[:cut % (len(b) + 1)]))
    _decode_safely(nat.decode_packet, bytes(b[:cut % (len(b) + 1)]))


@settings(max_examples=300, deadline=None)
@given(st.binary(max_size=256))
def test_random_bytes_never_crash(nat, b):
    for fn in (nat.decode_request, nat.decode_packet, nat.decode_hybrid_request):
        _decode_safely(fn, b)


def test_huge_declared_lengths_are_refused(nat):
    # shape of 2^60 dims, then a data length of 2^62 bytes: both beyond the buffer
    for blob in (struct.pack("<Q", 1 << 60) + b"\0" * 16,
                 struct.pack("<QQ", 1, 2) + struct.pack("<Q", 7) + b"float32" + b"\x01" + struct.pack("<Q", 1 << 62)):
        with pytest.raises((ValueError, RuntimeError)):
            nat.decode_packet(blob)
