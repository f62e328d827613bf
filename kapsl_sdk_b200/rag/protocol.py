"""RAG connector protocol: JSON lines over a sidecar's stdin/stdout.

Request:  ``{"id": ..., "method": <Method>, "params": {...}}`` (``params``
omitted for ``Health``).  Response: ``{"id": ..., "status": "Ok", "result":
{"type": <Result>, "value": ...}}`` or ``{"id": ..., "status": "Err",
"result": {"message": ..., "code": null}}``.  Methods: ValidateConfig,
AuthStart, AuthCallback, ListSources, Sync, FetchDocument, TransformPrompt,
ResolveAcl, Health; result types: Unit, AuthUrl, Sources, Deltas, Document,
PromptTransform, Acl, Health.  Enum values inside payloads are kebab-case.

The encoding follows the reference connector SDK's serde layout
(crates/kapsl-rag-sdk/src/protocol.rs:8-79, types.rs:1-64, manifest.rs:3-41)
so existing connectors interoperate.
"""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field
from typing import Any, Optional

METHODS = ("ValidateConfig", "AuthStart", "AuthCallback", "ListSources", "Sync", "FetchDocument",
           "TransformPrompt", "ResolveAcl", "Health")
RESULT_TYPES = ("Unit", "AuthUrl", "Sources", "Deltas", "Document", "PromptTransform", "Acl", "Health")
RUNTIMES = ("wasm", "sidecar")
CAPABILITIES = ("sync", "on-demand", "prompt-transform")
AUTH_METHODS = ("none", "api-key", "o-auth-device-code", "o-auth-authorization-code", "aws-access-key",
                "aws-assume-role")


@dataclass
class ExternalAcl:
    allow_users: list = field(default_factory=list)
    allow_groups: list = field(default_factory=list)
    deny_users: list = field(default_factory=list)
    deny_groups: list = field(default_factory=list)

    @classmethod
    def from_json(cls, d: Optional[dict]) -> "ExternalAcl":
        d = d or {}
        return cls(list(d.get("allow_users", [])), list(d.get("allow_groups", [])), list(d.get("deny_users", [])),
                   list(d.get("deny_groups", [])))


@dataclass
class SourceDescriptor:
    id: str
    name: str
    kind: str
    metadata: dict = field(default_factory=dict)


@dataclass
class DocumentDelta:
    id: str
    op: str  # "upsert" | "delete"
    etag: Optional[str] = None
    modified_at: Optional[str] = None
    metadata: dict = field(default_factory=dict)
    acl: ExternalAcl = field(default_factory=ExternalAcl)

    @classmethod
    def from_json(cls, d: dict) -> "DocumentDelta":
        if d["op"] not in ("upsert", "delete"):
            raise ValueError(f"unknown delta op {d['op']!r}")
        return cls(d["id"], d["op"], d.get("etag"), d.get("modified_at"), dict(d.get("metadata", {})),
                   ExternalAcl.from_json(d.get("acl")))


@dataclass
class DocumentPayload:
    id: str
    content_type: str
    bytes_b64: str
    metadata: dict = field(default_factory=dict)
    acl: ExternalAcl = field(default_factory=ExternalAcl)

    @classmethod
    def from_json(cls, d: dict) -> "DocumentPayload":
        return cls(d["id"], d["content_type"], d["bytes_b64"], dict(d.get("metadata", {})),
                   ExternalAcl.from_json(d.get("acl")))


@dataclass
class ConnectorManifest:
    id: str
    name: str
    version: str
    runtime: str
    capabilities: list
    auth: list
    permissions: list
    description: Optional[str] = None
    entrypoint: Optional[str] = None
    config_schema: Any = None

    @classmethod
    def from_json(cls, d: dict) -> "ConnectorManifest":
        m = cls(d["id"], d["name"], d["version"], d["runtime"], list(d["capabilities"]), list(d["auth"]),
                list(d["permissions"]), d.get("description"), d.get("entrypoint"), d.get("config_schema"))
        if m.runtime not in RUNTIMES:
            raise ValueError(f"unknown connector runtime {m.runtime!r}")
        for c in m.capabilities:
            if c not in CAPABILITIES:
                raise ValueError(f"unknown connector capability {c!r}")
        for a in m.auth:
            if a not in AUTH_METHODS:
                raise ValueError(f"unknown auth method {a!r}")
        return m


class ConnectorRemoteError(RuntimeError):
    def __init__(self, message: str, code: Optional[str] = None):
        super().__init__(message)
        self.code = code


def _to_json(v):
    if hasattr(v, "__dataclass_fields__"):
        return asdict(v)
    if isinstance(v, list):
        return [_to_json(x) for x in v]
    return v


def encode_request(req_id: str, method: str, params: Optional[dict] = None) -> str:
    if method not in METHODS:
        raise ValueError(f"unknown connector method {method!r}")
    msg = {"id": req_id, "method": method}
    if method != "Health":
        msg["params"] = {k: _to_json(v) for k, v in (params or {}).items()}
    return json.dumps(msg)


def decode_request(line: str) -> tuple:
    d = json.loads(line)
    method = d["method"]
    if method not in METHODS:
        raise ValueError(f"unknown connector method {method!r}")
    return d["id"], method, d.get("params") or {}


def encode_ok(req_id: str, rtype: str, value=None) -> str:
    if rtype not in RESULT_TYPES:
        raise ValueError(f"unknown result type {rtype!r}")
    result = {"type": rtype}
    if rtype != "Unit":
        result["value"] = _to_json(value)
    return json.dumps({"id": req_id, "status": "Ok", "result": result})


def encode_err(req_id: str, message: str, code: Optional[str] = None) -> str:
    return json.dumps({"id": req_id, "status": "Err", "result": {"message": message, "code": code}})


def decode_response(line: str) -> tuple:
    """-> (id, result type, decoded value); raises ConnectorRemoteError for Err responses."""
    d = json.loads(line)
    if d["status"] == "Err":
        r = d.get("result") or {}
        raise ConnectorRemoteError(r.get("message", ""), r.get("code"))
    r = d["result"]
    t = r["type"]
    v = r.get("value")
    if t == "Sources":
        v = [SourceDescriptor(x["id"], x["name"], x["kind"], dict(x.get("metadata", {}))) for x in v]
    elif t == "Deltas":
        v = [DocumentDelta.from_json(x) for x in v]
    elif t == "Document":
        v = DocumentPayload.from_json(v)
    elif t == "Acl":
        v = ExternalAcl.from_json(v)
    elif t == "PromptTransform":
        v = v["prompt"]
    return d["id"], t, v
