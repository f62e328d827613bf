"""Document store on the filesystem and a SQLite vector store with ACL filtering.

SQLite table ``rag_chunks`` keeps, per chunk: scope (tenant, workspace,
source, document), index, text, the embedding as little-endian float32
bytes, metadata JSON and four ACL lists (JSON arrays).  A query keeps the
chunks of the tenant/workspace (and optional sources) that pass the ACL
(allowed when the chunk has no allow lists or shares a user/group with them,
never when a deny list matches), scores them by cosine similarity and
returns the top k at or above ``min_score``.  Scoring is one matrix-vector
product over the candidate embeddings (torch; on the GPU when asked), not a
Python loop (reference: crates/kapsl-rag/src/vector/mod.rs:26-359 scores
row by row; storage/mod.rs:18-70 for the document store).
"""
from __future__ import annotations

import json
import os
import sqlite3
import threading
import time
from dataclasses import dataclass, field
from typing import Optional

import numpy as np


@dataclass
class DocKey:
    tenant_id: str
    workspace_id: str
    source_id: str
    doc_id: str


class FsDocStore:
    def __init__(self, root: str):
        self.root = root

    def _path(self, key: DocKey) -> str:
        parts = [key.tenant_id, key.workspace_id, key.source_id, key.doc_id]
        for p in parts:
            if not p or "/" in p or p in (".", ".."):
                raise ValueError(f"invalid document key component {p!r}")
        return os.path.join(self.root, *parts)

    def put(self, key: DocKey, data: bytes) -> str:
        p = self._path(key)
        os.makedirs(os.path.dirname(p), exist_ok=True)
        with open(p, "wb") as f:
            f.write(data)
        return p

    def get(self, key: DocKey) -> bytes:
        with open(self._path(key), "rb") as f:
            return f.read()

    def delete(self, key: DocKey) -> None:
        p = self._path(key)
        if os.path.exists(p):
            os.remove(p)


@dataclass
class AccessControl:
    allow_users: list = field(default_factory=list)
    allow_groups: list = field(default_factory=list)
    deny_users: list = field(default_factory=list)
    deny_groups: list = field(default_factory=list)


@dataclass
class EmbeddedChunk:
    id: str
    tenant_id: str
    workspace_id: str
    source_id: str
    doc_id: str
    chunk_index: int
    text: str
    embedding: list
    metadata: dict = field(default_factory=dict)
    acl: AccessControl = field(default_factory=AccessControl)


@dataclass
class VectorQuery:
    query_embedding: list
    top_k: int
    tenant_id: str
    workspace_id: str
    source_ids: Optional[list] = None
    allowed_users: list = field(default_factory=list)
    allowed_groups: list = field(default_factory=list)
    min_score: float = 0.0


@dataclass
class VectorSearchResult:
    chunk: EmbeddedChunk
    score: float


_SCHEMA = """
CREATE TABLE IF NOT EXISTS rag_chunks (
    id TEXT PRIMARY KEY, tenant_id TEXT NOT NULL, workspace_id TEXT NOT NULL, source_id TEXT NOT NULL,
    doc_id TEXT NOT NULL, chunk_index INTEGER NOT NULL, text TEXT NOT NULL, embedding BLOB NOT NULL,
    metadata_json TEXT, acl_allow_users TEXT, acl_allow_groups TEXT, acl_deny_users TEXT, acl_deny_groups TEXT,
    updated_at INTEGER);
CREATE INDEX IF NOT EXISTS idx_rag_chunks_scope ON rag_chunks (tenant_id, workspace_id, source_id, doc_id);
"""


def _allowed(users: set, groups: set, acl_users: list, acl_groups: list) -> bool:
    if not acl_users and not acl_groups:
        return True
    return any(u in users for u in acl_users) or any(g in groups for g in acl_groups)


def _denied(users: set, groups: set, deny_users: list, deny_groups: list) -> bool:
    return any(u in users for u in deny_users) or any(g in groups for g in deny_groups)


def _json_list(s: Optional[str]) -> list:
    try:
        v = json.loads(s) if s else []
    except ValueError:
        return []
    return [x for x in v if isinstance(x, str)] if isinstance(v, list) else []


class SqliteVectorStore:
    def __init__(self, path: str, device: str = "cpu"):
        self._conn = sqlite3.connect(path, check_same_thread=False)
        self._lock = threading.Lock()
        self.device = device
        with self._lock:
            self._conn.executescript(_SCHEMA)

    def upsert(self, chunks: list) -> None:
        rows = [(c.id, c.tenant_id, c.workspace_id, c.source_id, c.doc_id, int(c.chunk_index), c.text,
                 np.asarray(c.embedding, dtype="<f4").tobytes(), json.dumps(c.metadata),
                 json.dumps(c.acl.allow_users), json.dumps(c.acl.allow_groups), json.dumps(c.acl.deny_users),
                 json.dumps(c.acl.deny_groups), int(time.time())) for c in chunks]
        with self._lock:
            self._conn.executemany("INSERT OR REPLACE INTO rag_chunks VALUES (?,?,?,?,?,?,?,?,?,?,?,?,?,?)", rows)
            self._conn.commit()

    def delete_by_doc(self, tenant_id: str, workspace_id: str, source_id: str, doc_id: str) -> int:
        with self._lock:
            cur = self._conn.execute("DELETE FROM rag_chunks WHERE tenant_id=? AND workspace_id=? AND source_id=? "
                                     "AND doc_id=?", (tenant_id, workspace_id, source_id, doc_id))
            self._conn.commit()
            return cur.rowcount

    def query(self, q: VectorQuery) -> list:
        import torch

        if not q.query_embedding:
            raise ValueError("query embedding is empty")
        sql = ("SELECT id, tenant_id, workspace_id, source_id, doc_id, chunk_index, text, embedding, metadata_json, "
               "acl_allow_users, acl_allow_groups, acl_deny_users, acl_deny_groups FROM rag_chunks "
               "WHERE tenant_id = ? AND workspace_id = ?")
        args = [q.tenant_id, q.workspace_id]
        if q.source_ids:
            sql += " AND source_id IN (" + ", ".join("?" * len(q.source_ids)) + ")"
            args += list(q.source_ids)
        with self._lock:
            rows = self._conn.execute(sql, args).fetchall()
        users, groups = set(q.allowed_users), set(q.allowed_groups)
        dim = len(q.query_embedding)
        keep, embs = [], []
        for r in rows:
            e = np.frombuffer(r[7], dtype="<f4")
            if e.shape[0] != dim:
                continue
            acl = AccessControl(_json_list(r[9]), _json_list(r[10]), _json_list(r[11]), _json_list(r[12]))
            if not _allowed(users, groups, acl.allow_users, acl.allow_groups):
                continue
            if _denied(users, groups, acl.deny_users, acl.deny_groups):
                continue
            keep.append((r, acl))
            embs.append(e)
        if not keep:
            return []
        m = torch.from_numpy(np.stack(embs)).to(self.device)
        v = torch.tensor(q.query_embedding, dtype=torch.float32, device=self.device)
        norms = m.norm(dim=1) * v.norm()
        scores = torch.where(norms > 0, (m @ v) / norms.clamp_min(1e-30), torch.zeros_like(norms)).cpu().tolist()
        out = []
        for (r, acl), s, e in zip(keep, scores, embs):
            if s < q.min_score:
                continue
            meta = json.loads(r[8]) if r[8] else {}
            out.append(VectorSearchResult(EmbeddedChunk(r[0], r[1], r[2], r[3], r[4], r[5], r[6], e.tolist(), meta,
                                                        acl), float(s)))
        out.sort(key=lambda x: (-x.score, x.chunk.id))
        return out[:q.top_k]
