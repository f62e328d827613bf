"""Connector side of the protocol: subclass :class:`Connector` and call
:func:`serve_stdio` in the sidecar's ``main`` (reference:
crates/kapsl-rag-sdk/src/server.rs:41-140)."""
from __future__ import annotations

import sys
from typing import Optional, TextIO

from .protocol import (DocumentDelta, DocumentPayload, ExternalAcl, SourceDescriptor, decode_request, encode_err,
                       encode_ok)


class ConnectorError(Exception):
    """Error raised by a connector; ``kind`` prefixes the message sent back."""

    def __init__(self, kind: str, detail: str):
        super().__init__(f"{kind}: {detail}")


def unsupported(what: str) -> ConnectorError:
    return ConnectorError("unsupported operation", what)


class Connector:
    """Override what the connector supports; the defaults answer like the
    reference SDK (prompt transformation unsupported, health "ok")."""

    def validate_config(self, config) -> None:
        raise unsupported("validate_config")

    def auth_start(self, config) -> str:
        raise unsupported("auth")

    def auth_callback(self, code: str, state: Optional[str]) -> None:
        raise unsupported("auth")

    def list_sources(self, config) -> list:
        raise unsupported("list_sources")

    def sync(self, source_id: str, cursor: Optional[str]) -> list:
        raise unsupported("sync")

    def fetch_document(self, document_id: str) -> DocumentPayload:
        raise unsupported("fetch_document")

    def transform_prompt(self, config, prompt: str) -> str:
        raise unsupported("prompt transformation is not implemented")

    def resolve_acl(self, acl: ExternalAcl) -> ExternalAcl:
        return acl

    def health(self) -> str:
        return "ok"


def dispatch(connector: Connector, line: str) -> str:
    try:
        req_id, method, p = decode_request(line)
    except Exception as e:  # malformed request: answer with an error line, keep serving
        return encode_err("", f"serialization error: {e}")
    try:
        if method == "ValidateConfig":
            connector.validate_config(p.get("config"))
            return encode_ok(req_id, "Unit")
        if method == "AuthStart":
            return encode_ok(req_id, "AuthUrl", connector.auth_start(p.get("config")))
        if method == "AuthCallback":
            connector.auth_callback(p["code"], p.get("state"))
            return encode_ok(req_id, "Unit")
        if method == "ListSources":
            return encode_ok(req_id, "Sources", connector.list_sources(p.get("config")))
        if method == "Sync":
            return encode_ok(req_id, "Deltas", connector.sync(p["source_id"], p.get("cursor")))
        if method == "FetchDocument":
            return encode_ok(req_id, "Document", connector.fetch_document(p["document_id"]))
        if method == "TransformPrompt":
            return encode_ok(req_id, "PromptTransform", {"prompt": connector.transform_prompt(p.get("config"),
                                                                                         p["prompt"])})
        if method == "ResolveAcl":
            return encode_ok(req_id, "Acl", connector.resolve_acl(ExternalAcl.from_json(p.get("acl"))))
        return encode_ok(req_id, "Health", connector.health())
    except ConnectorError as e:
        return encode_err(req_id, str(e))
    except KeyError as e:
        return encode_err(req_id, f"invalid input: missing {e}")
    except Exception as e:
        return encode_err(req_id, f"internal error: {e}")


def serve_stdio(connector: Connector, stdin: TextIO = None, stdout: TextIO = None) -> None:
    """Answer one JSON line per request line until stdin closes."""
    stdin = stdin or sys.stdin
    stdout = stdout or sys.stdout
    for line in stdin:
        if not line.strip():
            continue
        stdout.write(dispatch(connector, line) + "\n")
        stdout.flush()


__all__ = ["Connector", "ConnectorError", "serve_stdio", "dispatch", "SourceDescriptor", "DocumentDelta",
           "DocumentPayload", "ExternalAcl"]
