"""Ingestion: parse -> chunk -> embed -> vector store.

* :class:`PlainTextParser` — base64 UTF-8 payloads.
* :class:`SimpleChunker` — whitespace tokens, windows of ``chunk_size`` with
  ``overlap`` tokens shared; chunk ids ``<doc>:<index>`` and a
  ``chunk_index`` metadata entry.
* :class:`DummyEmbedder` — zero vectors (the reference's placeholder);
  :class:`HashEmbedder` — deterministic feature hashing of lower-cased
  tokens, L2-normalised, so retrieval works without a model;
  :class:`ModelEmbedder` — mean-pooled hidden states of a loaded decoder.

Reference: crates/kapsl-rag/src/ingestion/mod.rs:45-203.
"""
from __future__ import annotations

import base64
import zlib
from dataclasses import dataclass, field

import numpy as np

from .protocol import DocumentPayload
from .store import AccessControl, EmbeddedChunk


@dataclass
class ParsedDocument:
    id: str
    text: str
    metadata: dict = field(default_factory=dict)
    content_type: str = "text/plain"


@dataclass
class Chunk:
    id: str
    index: int
    text: str
    metadata: dict = field(default_factory=dict)


class PlainTextParser:
    def parse(self, payload: DocumentPayload) -> ParsedDocument:
        try:
            text = base64.b64decode(payload.bytes_b64, validate=True).decode("utf-8")
        except Exception as e:
            raise ValueError(f"parse error: {e}") from e
        return ParsedDocument(payload.id, text, dict(payload.metadata), payload.content_type)


class SimpleChunker:
    def __init__(self, chunk_size: int = 200, overlap: int = 20):
        if chunk_size <= 0:
            raise ValueError("chunk_size must be positive")
        self.chunk_size, self.overlap = chunk_size, overlap

    def chunk(self, doc: ParsedDocument) -> list:
        toks = doc.text.split()
        out = []
        start, index = 0, 0
        while start < len(toks):
            end = min(start + self.chunk_size, len(toks))
            meta = dict(doc.metadata)
            meta["chunk_index"] = str(index)
            out.append(Chunk(f"{doc.id}:{index}", index, " ".join(toks[start:end]), meta))
            if end == len(toks):
                break
            start = max(end - min(self.overlap, self.chunk_size), start + 1)
            index += 1
        return out


class DummyEmbedder:
    def __init__(self, dimension: int = 384):
        self.dimension = dimension

    def embed(self, texts: list) -> list:
        return [[0.0] * self.dimension for _ in texts]


class HashEmbedder:
    def __init__(self, dimension: int = 256):
        self.dimension = dimension

    def embed(self, texts: list) -> list:
        out = np.zeros((len(texts), self.dimension), dtype=np.float32)
        for i, t in enumerate(texts):
            for w in t.lower().split():
                h = zlib.crc32(w.encode())
                out[i, h % self.dimension] += 1.0 if (h >> 31) & 1 else -1.0
        n = np.linalg.norm(out, axis=1, keepdims=True)
        return (out / np.where(n > 0, n, 1.0)).tolist()


class ModelEmbedder:
    """Mean of the final hidden states of a :class:`~kapsl_sdk_b200.models.cpu_model.CPUCausalLM`
    style model exposing ``embed_tokens(ids) -> [T, d]`` plus a tokenizer."""

    def __init__(self, embed_fn, tokenizer):
        self.embed_fn, self.tokenizer = embed_fn, tokenizer

    def embed(self, texts: list) -> list:
        out = []
        for t in texts:
            h = np.asarray(self.embed_fn(self.tokenizer.encode(t)), dtype=np.float32).mean(0)
            out.append((h / max(float(np.linalg.norm(h)), 1e-12)).tolist())
        return out


@dataclass
class IngestionContext:
    tenant_id: str
    workspace_id: str
    source_id: str
    acl: AccessControl = field(default_factory=AccessControl)


class IngestionPipeline:
    def __init__(self, parser, chunker, embedder, vector_store):
        self.parser, self.chunker, self.embedder, self.store = parser, chunker, embedder, vector_store

    def ingest(self, ctx: IngestionContext, payload: DocumentPayload) -> int:
        """Replace the document's chunks in the store; returns the number of chunks written."""
        doc = self.parser.parse(payload)
        chunks = self.chunker.chunk(doc)
        self.store.delete_by_doc(ctx.tenant_id, ctx.workspace_id, ctx.source_id, doc.id)
        if not chunks:
            return 0
        embs = self.embedder.embed([c.text for c in chunks])
        acl = ctx.acl
        if payload.acl is not None and (payload.acl.allow_users or payload.acl.allow_groups or
                                        payload.acl.deny_users or payload.acl.deny_groups):
            a = payload.acl
            acl = AccessControl(a.allow_users, a.allow_groups, a.deny_users, a.deny_groups)
        self.store.upsert([EmbeddedChunk(c.id, ctx.tenant_id, ctx.workspace_id, ctx.source_id, doc.id, c.index, c.text,
                                         e, c.metadata, acl) for c, e in zip(chunks, embs)])
        return len(chunks)
