"""Document store on the filesystem and a SQLite vector store with ACL filtering.

SQLite table ``rag_chunks`` keeps, per chunk: scope (tenant, workspace,
source, document), index, text, the embedding as little-endian float32
bytes, metadata JSON and four ACL lists (JSON arrays).  A query keeps the
chunks of the tenant/workspace (and optional sources) that pass the ACL
(allowed when the chunk has no allow lists or shares a user/group with them,
never when a deny list matches), scores them by cosine similarity and
returns the top k at or above ``min_score``.  Scoring is one matrix-vector
product over the candidate embeddings (torch; on the GPU when asked), not a
Python loop, over rows kept resident after the first query, or an HNSW
graph search for large scopes (reference: crates/kapsl-rag/src/vector/mod.rs:26-359
reads and scores every row per query; storage/mod.rs:18-70 for the document store).
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
    if not s or s == "[]":
        return []
    try:
        v = json.loads(s) if s else []
    except ValueError:
        return []
    return [x for x in v if isinstance(x, str)] if isinstance(v, list) else []


class _Scope:
    """Resident copy of one (tenant, workspace): unit-norm embeddings per row,
    row fields, ACLs, an alive mask (deleted or replaced rows stay as dead
    rows) and, when asked for, an HNSW graph whose labels are the row numbers."""

    def __init__(self, dim: int, use_hnsw: bool):
        from .. import _native

        self.dim = dim
        self.rows, self.acls, self.sources, self.raw, self.pos = [], [], [], [], {}
        self.emb = np.zeros((0, dim), np.float32)
        self.alive = np.zeros(0, bool)
        self.public = np.zeros(0, bool)  # no allow and no deny lists
        self.hnsw = _native.rag.Hnsw(dim) if use_hnsw else None
        self._pending = []
        self._dev = None  # (device, tensor) copy of emb for flat scoring

    def tensor(self, device: str):
        import torch

        if self._dev is None or self._dev[0] != device:
            self._dev = (device, torch.from_numpy(self.emb).to(device))
        return self._dev[1]

    def add(self, row: tuple, acl: AccessControl, emb: np.ndarray, pending: bool = True) -> None:
        """One row; with ``pending=False`` the caller queues its embedding as
        part of a matrix (``add_matrix``)."""
        old = self.pos.get(row[0])
        if old is not None:
            self.kill(old)
        n = len(self.rows)
        self.pos[row[0]] = n
        self.rows.append(row)
        self.acls.append(acl)
        self.sources.append(row[3])
        self.raw.append(emb)
        if pending:
            self.add_matrix(emb[None], np.array([self._public(acl)]))

    @staticmethod
    def _public(acl: AccessControl) -> bool:
        return not (acl.allow_users or acl.allow_groups or acl.deny_users or acl.deny_groups)

    def add_matrix(self, emb: np.ndarray, public: np.ndarray) -> None:
        self._pending.append((emb, public))

    def flush(self) -> None:
        if not self._pending:
            return
        e = np.concatenate([m for m, _ in self._pending]).astype(np.float32)
        pub = np.concatenate([p for _, p in self._pending])
        norm = np.linalg.norm(e, axis=1, keepdims=True)
        e = np.divide(e, norm, out=np.zeros_like(e), where=norm > 0)  # zero rows stay zero (score 0)
        self.emb = np.concatenate([self.emb, e])
        self._dev = None
        self.alive = np.concatenate([self.alive, np.ones(len(e), bool)])
        self.public = np.concatenate([self.public, pub.astype(bool)])
        if self.hnsw is not None:  # rows a loaded graph already holds are not inserted again
            skip = max(0, len(self.hnsw) - (len(self.alive) - len(e)))
            if skip < len(e):
                self.hnsw.add(e[skip:])
        self._pending = []

    def kill(self, n: int) -> None:
        self.flush()
        self.alive[n] = False
        if self.hnsw is not None:
            self.hnsw.remove(n)


class SqliteVectorStore:
    """``index="flat"`` scores every candidate row with one matrix-vector product
    (torch, on ``device``); ``index="hnsw"`` searches an HNSW graph
    (``_native.rag.Hnsw``) when more than ``exact_below`` rows pass the filters,
    and scores exactly below that.  Rows stay resident per (tenant, workspace)
    after the first query; writes through this object update that copy, and a
    commit by another connection (SQLite's ``data_version``) drops it."""

    def __init__(self, path: str, device: str = "cpu", index: str = "flat", ef_search: int = 96,
                 exact_below: int = 4096, index_dir: Optional[str] = None):
        """``index_dir``: with ``index="hnsw"``, graphs are saved there and loaded
        again by a later store whose scope holds the same rows (same ids and
        update times in rowid order), instead of being rebuilt."""
        if index not in ("flat", "hnsw"):
            raise ValueError(f"unknown vector index {index!r}")
        self.index_dir = index_dir
        self._conn = sqlite3.connect(path, check_same_thread=False)
        self._lock = threading.Lock()
        self.device, self.index, self.ef_search, self.exact_below = device, index, ef_search, exact_below
        self._scopes: dict = {}
        with self._lock:
            self._conn.executescript(_SCHEMA)
            self._version = self._data_version()

    def _data_version(self) -> int:
        return self._conn.execute("PRAGMA data_version").fetchone()[0]

    def _check_version(self) -> None:
        v = self._data_version()
        if v != self._version:  # another connection committed
            self._scopes.clear()
            self._version = v

    def upsert(self, chunks: list) -> None:
        rows = [(c.id, c.tenant_id, c.workspace_id, c.source_id, c.doc_id, int(c.chunk_index), c.text,
                 np.asarray(c.embedding, dtype="<f4").tobytes(), json.dumps(c.metadata),
                 json.dumps(c.acl.allow_users), json.dumps(c.acl.allow_groups), json.dumps(c.acl.deny_users),
                 json.dumps(c.acl.deny_groups), int(time.time())) for c in chunks]
        with self._lock:
            self._check_version()
            self._conn.executemany("INSERT OR REPLACE INTO rag_chunks VALUES (?,?,?,?,?,?,?,?,?,?,?,?,?,?)", rows)
            self._conn.commit()
            for r in rows:
                self._mirror_row(r)

    def _mirror_row(self, r: tuple) -> None:
        for key in list(self._scopes):
            if key[:2] != (r[1], r[2]):
                continue
            sc = self._scopes[key]
            old = sc.pos.pop(r[0], None)
            if old is not None:
                sc.kill(old)
            e = np.frombuffer(r[7], dtype="<f4")
            if e.shape[0] == sc.dim:
                sc.add(r[:7] + r[8:9], AccessControl(_json_list(r[9]), _json_list(r[10]), _json_list(r[11]),
                                                     _json_list(r[12])), e)

    def delete_by_doc(self, tenant_id: str, workspace_id: str, source_id: str, doc_id: str) -> int:
        with self._lock:
            self._check_version()
            cur = self._conn.execute("DELETE FROM rag_chunks WHERE tenant_id=? AND workspace_id=? AND source_id=? "
                                     "AND doc_id=?", (tenant_id, workspace_id, source_id, doc_id))
            self._conn.commit()
            for key, sc in self._scopes.items():
                if key[:2] != (tenant_id, workspace_id):
                    continue
                for n, row in enumerate(sc.rows):
                    if row[3] == source_id and row[4] == doc_id and sc.pos.get(row[0]) == n:
                        del sc.pos[row[0]]
                        sc.kill(n)
            return cur.rowcount

    def _scope(self, tenant_id: str, workspace_id: str, dim: int) -> _Scope:
        key = (tenant_id, workspace_id, dim)
        sc = self._scopes.get(key)
        if sc is None:
            sc = _Scope(dim, self.index == "hnsw")
            rows = self._conn.execute(
                "SELECT id, tenant_id, workspace_id, source_id, doc_id, chunk_index, text, embedding, metadata_json, "
                "acl_allow_users, acl_allow_groups, acl_deny_users, acl_deny_groups, updated_at FROM rag_chunks "
                "WHERE tenant_id = ? AND workspace_id = ? ORDER BY rowid", (tenant_id, workspace_id)).fetchall()
            rows = [r for r in rows if len(r[7]) == 4 * dim]
            cache = self._graph_path(tenant_id, workspace_id, dim, rows) if sc.hnsw is not None else None
            if cache is not None and os.path.exists(cache):
                from .. import _native

                try:
                    g = _native.rag.Hnsw.load(cache)
                    if len(g) == len(rows) and g.dim == dim:
                        sc.hnsw = g
                except (RuntimeError, ValueError):
                    pass  # unreadable: rebuilt and saved again below
            emb = np.frombuffer(b"".join(r[7] for r in rows), dtype="<f4").reshape(len(rows), dim)
            pub = np.zeros(len(rows), bool)
            for i, (r, e) in enumerate(zip(rows, emb)):
                acl = AccessControl(_json_list(r[9]), _json_list(r[10]), _json_list(r[11]), _json_list(r[12]))
                sc.add(r[:7] + r[8:9], acl, e, pending=False)
                pub[i] = sc._public(acl)
            sc.add_matrix(emb, pub)
            self._scopes[key] = sc
            if cache is not None:
                rebuilt = len(sc.hnsw) < len(rows)
                sc.flush()
                if rebuilt:
                    self._save_graph(sc.hnsw, cache)
        sc.flush()
        return sc

    def _graph_path(self, tenant_id: str, workspace_id: str, dim: int, rows: list) -> Optional[str]:
        if not self.index_dir:
            return None
        import hashlib

        scope = hashlib.sha1(f"{tenant_id}\0{workspace_id}\0{dim}".encode()).hexdigest()[:16]
        # the key covers each row's id, update time AND embedding bytes: an
        # upsert within the same second keeps id, time and row order, so only
        # the vector itself tells a stale graph from a current one
        h = hashlib.sha1()
        for r in rows:
            h.update(f"{r[0]}\0{r[13]}\n".encode())
            h.update(r[7])
        return os.path.join(self.index_dir, f"{scope}-{h.hexdigest()[:24]}.hnsw")

    @staticmethod
    def _save_graph(g, path: str) -> None:
        d = os.path.dirname(path)
        os.makedirs(d, exist_ok=True)
        tmp = f"{path}.{os.getpid()}.tmp"
        g.save(tmp)
        os.replace(tmp, path)
        prefix = os.path.basename(path).split("-")[0] + "-"
        for f in os.listdir(d):  # older graphs of the same scope
            if f.startswith(prefix) and f.endswith(".hnsw") and os.path.join(d, f) != path:
                try:
                    os.remove(os.path.join(d, f))
                except OSError:
                    pass

    def query(self, q: VectorQuery) -> list:
        import torch

        if not q.query_embedding:
            raise ValueError("query embedding is empty")
        v = np.asarray(q.query_embedding, dtype=np.float32)
        with self._lock:
            self._check_version()
            sc = self._scope(q.tenant_id, q.workspace_id, v.shape[0])
            n = len(sc.rows)
            if n == 0:
                return []
            mask = sc.alive & sc.public
            users, groups = set(q.allowed_users), set(q.allowed_groups)
            for i in np.flatnonzero(sc.alive & ~sc.public):
                a = sc.acls[i]
                mask[i] = _allowed(users, groups, a.allow_users, a.allow_groups) and \
                    not _denied(users, groups, a.deny_users, a.deny_groups)
            if q.source_ids:
                mask &= np.isin(np.asarray(sc.sources, dtype=object), list(q.source_ids))
            cand = np.flatnonzero(mask)
            if len(cand) == 0:
                return []
            vn = float(np.linalg.norm(v))
            if sc.hnsw is not None and len(cand) > self.exact_below and vn > 0:
                k = q.top_k
                while True:  # widen the beam until k rows pass the filter (or no more can)
                    s, lab = sc.hnsw.search(v, k, max(self.ef_search, k), mask.view(np.uint8))
                    if len(lab) >= q.top_k or k >= len(cand):
                        break
                    k *= 4
                idx, scores = lab[:q.top_k], s[:q.top_k].astype(np.float64).tolist()
            else:
                sims = sc.tensor(self.device) @ torch.from_numpy(v).to(self.device)
                sims = sims / vn if vn > 0 else torch.zeros_like(sims)
                sims = sims.masked_fill(~torch.from_numpy(mask).to(self.device), float("-inf"))
                kth = torch.topk(sims, min(q.top_k, len(cand))).values[-1]
                keep = torch.nonzero(sims >= kth).flatten()  # the k best and every row tied with the k-th
                sims, cand = sims[keep], keep.cpu().numpy()
                idx, scores = cand, sims.cpu().tolist()
            rows = [(sc.rows[i], sc.acls[i], sc.raw[i]) for i in idx]
        out = []
        for (r, acl, e), s in zip(rows, scores):
            if s < q.min_score:
                continue
            e = e.tolist()
            meta = json.loads(r[7]) if r[7] else {}
            out.append(VectorSearchResult(EmbeddedChunk(r[0], r[1], r[2], r[3], r[4], r[5], r[6], e, meta, acl),
                                          float(s)))
        out.sort(key=lambda x: (-x.score, x.chunk.id))
        return out[:q.top_k]
