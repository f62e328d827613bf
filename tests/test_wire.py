"""bincode wire codec: golden bytes hand-derived from the encoding rules, the
C++ codec against the pure-Python statement, and the decoder fallbacks."""
import base64
import struct

import pytest

from kapsl_sdk_b200.server import wire as pyw


@pytest.fixture(scope="module")
def nat():
    from kapsl_sdk_b200._ext import native

    return native()


def test_packet_golden_bytes(nat):
    data = struct.pack("<3f", 1.0, 2.0, 3.0)
    expect = (
        b"\x02\x00\x00\x00\x00\x00\x00\x00"          # shape len 2
        b"\x01\x00\x00\x00\x00\x00\x00\x00"          # 1
        b"\x03\x00\x00\x00\x00\x00\x00\x00"          # 3
        b"\x07\x00\x00\x00\x00\x00\x00\x00float32"   # dtype string
        b"\x01" b"\x0c\x00\x00\x00\x00\x00\x00\x00" + data +  # data: Some(12 bytes)
        b"\x00"                                       # data_base64: None
    )
    assert pyw.encode_packet([1, 3], "float32", data) == expect
    assert nat.encode_packet([1, 3], "float32", data) == expect
    assert nat.decode_packet(expect) == ([1, 3], "float32", data)


def test_request_with_auth_matches_python(nat):
    req = {"input": ([1, 5], "string", b"hello"), "additional_inputs": [("mask", ([2], "int64", b"\0" * 16))],
           "session_id": "s1", "metadata": {"auth_token": "tok"}}
    b_c = nat.encode_request(req)
    b_py = pyw.encode_request(([1, 5], "string", b"hello"), [("mask", ([2], "int64", b"\0" * 16))], "s1",
                              {"auth_token": "tok"})
    assert b_c == b_py
    # metadata: 5 None tags, auth Some("tok"), 7 None tags
    tail = b"\x01" + b"\x00" * 5 + b"\x01" + struct.pack("<Q", 3) + b"tok" + b"\x00" * 7
    assert b_c.endswith(tail)
    d = nat.decode_request(b_c)
    assert d["input"] == ([1, 5], "string", b"hello")
    assert d["session_id"] == "s1"
    assert d["metadata"]["auth_token"] == "tok"
    assert d["additional_inputs"][0][0] == "mask"


def test_full_metadata_roundtrip(nat):
    md = {"request_id": "r-1", "timeout_ms": 5000, "priority": 2, "force_cpu": True, "model_version": "v2",
          "auth_token": "t", "max_new_tokens": 64, "temperature": 0.5, "top_p": 0.75, "top_k": 7,
          "repetition_penalty": 1.25, "seed": 42, "stop_token_ids": [1, 2, 3]}
    req = {"input": ([2], "int32", b"\x01\0\0\0\x02\0\0\0"), "metadata": md}
    b = nat.encode_request(req)
    assert b == pyw.encode_request(([2], "int32", b"\x01\0\0\0\x02\0\0\0"), metadata=md)
    got = nat.decode_request(b)["metadata"]
    for k, v in md.items():
        assert got[k] == pytest.approx(v) if isinstance(v, float) else got[k] == v


def test_metadata_without_auth_and_legacy_layouts(nat):
    # auth_token omitted from the wire (skip_serializing_if) -> second layout
    md = {"request_id": "x", "max_new_tokens": 9}
    b = pyw.encode_request(([1], "uint8", b"\x07"), metadata=md)
    d = nat.decode_request(b)
    assert d["metadata"]["max_new_tokens"] == 9 and d["metadata"]["auth_token"] is None
    # legacy {input, additional_inputs, session_id}: no metadata field at all
    legacy = pyw.encode_packet([1], "uint8", b"\x07") + struct.pack("<Q", 0) + b"\x01" + \
        struct.pack("<Q", 2) + b"ab"
    d = nat.decode_request(legacy)
    assert d["session_id"] == "ab" and d["metadata"] is None


def test_base64_data_and_errors(nat):
    raw = b"\x01\x02\x03\x04"
    enc = base64.b64encode(raw)
    pkt = struct.pack("<Q", 1) + struct.pack("<q", 4) + struct.pack("<Q", 5) + b"uint8" + b"\x00" + b"\x01" + \
        struct.pack("<Q", len(enc)) + enc
    assert nat.decode_packet(pkt) == ([4], "uint8", raw)
    both = struct.pack("<Q", 0) + struct.pack("<Q", 5) + b"uint8" + b"\x01" + struct.pack("<Q", 0) + b"\x01" + \
        struct.pack("<Q", 0)
    with pytest.raises(ValueError):
        nat.decode_packet(both)
    with pytest.raises(ValueError):
        nat.decode_packet(b"\x01\x00")  # truncated


def test_dtype_aliases_and_validation(nat):
    assert nat.decode_packet(pyw.encode_packet([1], "FP32", b"\0" * 4))[1] == "float32"
    assert nat.validate_packet([2, 2], "float32", b"\0" * 16) == ""
    msg = nat.validate_packet([2, 2], "float32", b"\0" * 15)
    assert msg == "Data length mismatch: expected 16 bytes (4 float32 values) but got 15 bytes"
    assert nat.validate_packet([0, 2], "int32", b"") == "Invalid shape dimension: 0"


def test_frames_and_hybrid(nat):
    assert nat.request_header(3, 2, 17) == struct.pack("<III", 3, 2, 17)
    assert nat.response_header(1, 0) == b"\x01\0\0\0\0\0\0\0"
    h = {"request_id": 11, "model_id": 2, "priority": 1, "force_cpu": True, "timestamp_ns": 99,
         "shm_offset": 131072, "shm_size": 96}
    b = nat.encode_hybrid_request(h)
    # 24-byte #[repr(C)] RequestMetadata + two u64
    assert b == struct.pack("<QIBB2xQ", 11, 2, 1, 1, 99) + struct.pack("<QQ", 131072, 96)
    assert nat.decode_hybrid_request(b) == h
