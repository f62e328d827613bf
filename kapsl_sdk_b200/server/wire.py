"""Pure-Python statement of the bincode-1.3 wire encoding (legacy config).

The serving path uses the C++ codec in ``kapsl_sdk_b200._native``; this module
restates the same rules in Python so tests can cross-check the two and so the
format is readable in one place:

* fixed-width little-endian integers; ``u64`` length prefix for Vec/String/bytes;
* ``Option`` = 1-byte tag (0/1) then the value; ``bool`` = 1 byte;
* structs are their fields in declaration order;
* ``RequestMetadata.auth_token`` is skipped entirely when None
  (``skip_serializing_if``), which shifts the later fields.

Layouts: crates/kapsl-engine-api/src/lib.rs:272-339 (BinaryTensorPacket: shape,
dtype string, data Option<bytes> = Some, data_base64 Option<str> = None),
462-492 (RequestMetadata), 521-532 (InferenceRequest); frames in
crates/kapsl-ipc/src/protocol.rs.
"""
from __future__ import annotations

import struct
from typing import Optional

OP_INFER, OP_INFER_STREAM, OP_METRICS, OP_HYBRID_INFER = 1, 2, 3, 4
STATUS_OK, STATUS_ERR, STATUS_STREAM_CHUNK, STATUS_STREAM_END = 0, 1, 2, 3

META_FIELDS = [
    ("request_id", "str"), ("timeout_ms", "u64"), ("priority", "u8"), ("force_cpu", "bool"),
    ("model_version", "str"), ("auth_token", "str"), ("max_new_tokens", "u32"), ("temperature", "f32"),
    ("top_p", "f32"), ("top_k", "u32"), ("repetition_penalty", "f32"), ("seed", "u64"),
    ("stop_token_ids", "vec_u32"),
]


def _bytes(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def _scalar(kind: str, v) -> bytes:
    if kind == "str":
        return _bytes(v.encode())
    if kind == "u64":
        return struct.pack("<Q", v)
    if kind == "u32":
        return struct.pack("<I", v)
    if kind == "u8":
        return struct.pack("<B", v)
    if kind == "bool":
        return b"\x01" if v else b"\x00"
    if kind == "f32":
        return struct.pack("<f", v)
    if kind == "vec_u32":
        return struct.pack("<Q", len(v)) + b"".join(struct.pack("<I", x) for x in v)
    raise ValueError(kind)


def encode_packet(shape, dtype: str, data: bytes) -> bytes:
    out = struct.pack("<Q", len(shape)) + b"".join(struct.pack("<q", d) for d in shape)
    out += _bytes(dtype.encode())
    out += b"\x01" + _bytes(bytes(data))  # data: Some
    out += b"\x00"                        # data_base64: None
    return out


def encode_metadata(md: dict) -> bytes:
    out = b""
    for name, kind in META_FIELDS:
        v = md.get(name)
        if name == "auth_token" and v is None:
            continue  # skip_serializing_if = "Option::is_none"
        out += b"\x00" if v is None else b"\x01" + _scalar(kind, v)
    return out


def encode_request(input_packet: tuple, additional_inputs=(), session_id: Optional[str] = None,
                   metadata: Optional[dict] = None) -> bytes:
    out = encode_packet(*input_packet)
    out += struct.pack("<Q", len(additional_inputs))
    for name, pkt in additional_inputs:
        out += _bytes(name.encode()) + encode_packet(*pkt)
    out += b"\x00" if session_id is None else b"\x01" + _bytes(session_id.encode())
    out += b"\x00" if metadata is None else b"\x01" + encode_metadata(metadata)
    return out


def request_header(model_id: int, op: int, size: int) -> bytes:
    return struct.pack("<III", model_id, op, size)


def response_header(status: int, size: int) -> bytes:
    return struct.pack("<II", status, size)
