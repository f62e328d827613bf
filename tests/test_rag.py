"""RAG: connector JSON-lines protocol, a sidecar connector installed as an
extension, ingestion into the SQLite vector store, ACL-filtered queries and
prompt assembly."""
import base64
import json
import os
import sys
import textwrap

import numpy as np
import pytest

from kapsl_sdk_b200 import rag
from kapsl_sdk_b200.rag import protocol as P

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CONNECTOR = textwrap.dedent("""
    import base64, os, sys
    sys.path.insert(0, {root!r})
    from kapsl_sdk_b200.rag import Connector, ConnectorError, serve_stdio
    from kapsl_sdk_b200.rag.protocol import DocumentDelta, DocumentPayload, ExternalAcl, SourceDescriptor
    DOCS = {{
        "a": ("The B200 has 148 SMs and 180 GB of HBM3e memory.", ExternalAcl()),
        "b": ("NVLink 5 gives 900 GB/s per direction per GPU.", ExternalAcl(allow_groups=["eng"])),
        "c": ("Secret roadmap text that only admins may read.", ExternalAcl(allow_users=["alice"],
                                                                            deny_groups=["contractors"])),
    }}
    class Docs(Connector):
        def validate_config(self, config):
            if not isinstance(config, dict) or "root" not in config:
                raise ConnectorError("invalid input", "config needs 'root'")
        def list_sources(self, config):
            return [SourceDescriptor("kb", "Knowledge base", "folder", {{"owner": os.environ.get("OWNER", "")}})]
        def sync(self, source_id, cursor):
            return [DocumentDelta(k, "upsert", None, None, {{"source": "kb", "title": "doc-" + k}}, acl)
                    for k, (_, acl) in DOCS.items()]
        def fetch_document(self, document_id):
            text, acl = DOCS[document_id]
            return DocumentPayload(document_id, "text/plain", base64.b64encode(text.encode()).decode(),
                                   {{"source": "kb", "title": "doc-" + document_id}}, acl)
    serve_stdio(Docs())
""")


def test_protocol_encoding():
    line = P.encode_request("1", "Sync", {"source_id": "s", "cursor": None})
    assert json.loads(line) == {"id": "1", "method": "Sync", "params": {"source_id": "s", "cursor": None}}
    assert json.loads(P.encode_request("2", "Health")) == {"id": "2", "method": "Health"}
    assert json.loads(P.encode_ok("3", "Unit")) == {"id": "3", "status": "Ok", "result": {"type": "Unit"}}
    assert P.decode_response(P.encode_ok("4", "Health", "ok")) == ("4", "Health", "ok")
    with pytest.raises(P.ConnectorRemoteError, match="boom"):
        P.decode_response(P.encode_err("5", "boom"))
    with pytest.raises(ValueError):
        P.encode_request("6", "Nope")


def test_sidecar_extension_ingest_query_prompt(tmp_path):
    src = tmp_path / "src"
    src.mkdir()
    (src / "connector.py").write_text(CONNECTOR.format(root=ROOT))
    (src / "manifest.json").write_text(json.dumps({
        "id": "docs", "name": "Docs", "version": "0.1.0", "runtime": "sidecar", "capabilities": ["sync"],
        "auth": ["none"], "permissions": [], "entrypoint": "connector.py"}))
    reg = rag.ExtensionRegistry(str(tmp_path / "ext"))
    reg.install_from_dir(str(src))
    assert [e.id for e in reg.discover()] == ["docs"]
    mgr = rag.ExtensionManager(reg, str(tmp_path / "cfg"))
    mgr.set_workspace_config("ws1", "docs", {"root": "/data", "env": {"OWNER": "team"}})
    assert mgr.list_configs("ws1") == ["docs"]
    client = mgr.launch_connector("ws1", "docs")
    try:
        assert client.health() == "ok"
        client.validate_config({"root": "/data"})
        with pytest.raises(P.ConnectorRemoteError, match="invalid input"):
            client.validate_config({})
        with pytest.raises(P.ConnectorRemoteError, match="unsupported operation"):
            client.transform_prompt({}, "hi")
        (source,) = client.list_sources({"root": "/data"})
        assert source.id == "kb" and source.metadata["owner"] == "team"
        deltas = client.sync("kb")
        store = rag.SqliteVectorStore(str(tmp_path / "v.db"))
        pipe = rag.IngestionPipeline(rag.PlainTextParser(), rag.SimpleChunker(6, 2), rag.HashEmbedder(128), store)
        ctx = rag.IngestionContext("t", "ws1", "kb")
        docs = rag.FsDocStore(str(tmp_path / "docs"))
        n = 0
        for d in deltas:
            payload = client.fetch_document(d.id)
            docs.put(rag.DocKey("t", "ws1", "kb", d.id), base64.b64decode(payload.bytes_b64))
            n += pipe.ingest(ctx, payload)
        assert n >= 3
        assert docs.get(rag.DocKey("t", "ws1", "kb", "a")).startswith(b"The B200")
    finally:
        client.shutdown()

    emb = rag.HashEmbedder(128)
    q = emb.embed(["HBM3e memory SMs"])[0]
    anon = store.query(rag.VectorQuery(q, 10, "t", "ws1"))
    assert {r.chunk.doc_id for r in anon} == {"a"}  # b needs group eng, c needs alice
    eng = store.query(rag.VectorQuery(q, 10, "t", "ws1", allowed_groups=["eng"]))
    assert {r.chunk.doc_id for r in eng} == {"a", "b"}
    alice = store.query(rag.VectorQuery(q, 10, "t", "ws1", allowed_users=["alice"]))
    assert "c" in {r.chunk.doc_id for r in alice}
    contractor = store.query(rag.VectorQuery(q, 10, "t", "ws1", allowed_users=["alice"],
                                             allowed_groups=["contractors"]))
    assert "c" not in {r.chunk.doc_id for r in contractor}
    assert anon[0].score >= anon[-1].score and anon[0].chunk.doc_id == "a"
    assert store.query(rag.VectorQuery(q, 10, "other", "ws1")) == []

    chunks = [rag.RagChunk(r.chunk.id, r.chunk.text, r.score, r.chunk.metadata) for r in eng]
    p = rag.build_rag_prompt(chunks, rag.RagPromptConfig(max_per_source=2))
    assert p.context.startswith("[1] ") and "Source: doc-" in p.context and len(p.citations) == 2


def test_prompt_rules():
    C = rag.RagChunk
    chunks = [C("x1", "alpha beta gamma", 0.9, {"source": "s1"}), C("x2", "Alpha  BETA gamma", 0.8, {"source": "s2"}),
              C("x3", "delta epsilon", 0.7, {"source": "s1"}), C("x4", "zeta eta theta", 0.6, {"source": "s1"}),
              C("x5", "low", -1.0, {})]
    p = rag.build_rag_prompt(chunks, rag.RagPromptConfig(max_context_tokens=4, max_per_source=2))
    assert [c.chunk_id for c in p.citations] == ["x1", "x3"]  # x2 duplicate text, x4 over the per-source cap
    assert p.context == "[1] alpha beta gamma\nSource: s1\n\n[2] delta\nSource: s1"
    assert p.truncated and p.total_context_tokens == 4
    q = rag.build_rag_prompt(chunks[:1], rag.RagPromptConfig(citation_style="inline"))
    assert q.context == "alpha beta gamma (1)\nSource: s1"
    e = rag.build_rag_prompt([chunks[-1]])
    assert e.context == "" and e.fallback_message == "No relevant documents found."


def test_chunker():
    doc = rag.ParsedDocument("d", " ".join(str(i) for i in range(10)))
    cs = rag.SimpleChunker(4, 1).chunk(doc)
    assert [c.text for c in cs] == ["0 1 2 3", "3 4 5 6", "6 7 8 9"] and cs[1].id == "d:1"
    assert cs[2].metadata["chunk_index"] == "2"


def _clustered(n, dim, seed):
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((40, dim)).astype(np.float32)
    return (centers[rng.integers(0, 40, n)] + 0.6 * rng.standard_normal((n, dim))).astype(np.float32), centers


def test_hnsw_recall_filter_and_removal():
    from kapsl_sdk_b200 import _native

    X, centers = _clustered(6000, 48, 0)
    h = _native.rag.Hnsw(48, M=16, ef_construction=200, seed=7)
    assert list(h.add(X[:10])) == list(range(10)) and len(h.add(X[10:])) == 5990 and len(h) == 6000
    Xn = X / np.linalg.norm(X, axis=1, keepdims=True)
    rng = np.random.default_rng(1)
    hits = 0
    for _ in range(100):
        q = centers[rng.integers(0, 40)] + 0.6 * rng.standard_normal(48).astype(np.float32)
        s, lab = h.search(q, 10, 96)
        sims = Xn @ (q / np.linalg.norm(q))
        hits += len(set(lab.tolist()) & set(np.argsort(-sims)[:10].tolist()))
        assert np.allclose(s, sims[lab], atol=1e-5) and np.all(np.diff(s) <= 1e-6)
    assert hits / 1000 >= 0.95
    mask = np.zeros(6000, np.uint8)
    mask[::7] = 1  # filter: only every 7th label may be returned
    s, lab = h.search(X[3], 10, 400, mask)
    assert len(lab) == 10 and all(int(x) % 7 == 0 for x in lab)
    best = int(h.search(X[5], 1, 64)[1][0])
    h.remove(best)
    assert best not in h.search(X[5], 10, 64)[1].tolist()


@pytest.mark.parametrize("index", ["flat", "hnsw"])
def test_resident_store_matches_exact_scores_and_sees_other_writers(tmp_path, index):
    X, _ = _clustered(3000, 32, 2)
    db = str(tmp_path / "v.db")
    store = rag.SqliteVectorStore(db, index=index, exact_below=100)
    acl_eng = rag.AccessControl(allow_groups=["eng"])
    chunks = [rag.EmbeddedChunk(f"c{i}", "t", "ws", "src" + str(i % 3), f"d{i // 10}", i % 10, f"text {i}",
                                X[i].tolist(), {"i": i}, acl_eng if i % 5 == 0 else rag.AccessControl())
              for i in range(len(X))]
    store.upsert(chunks[:2000])
    q = X[17] + 0.1
    Xn = X / np.linalg.norm(X, axis=1, keepdims=True)

    def exact(n, allow_eng, sources=None):
        sims = Xn[:n] @ (q / np.linalg.norm(q))
        ok = [i for i in range(n) if (allow_eng or i % 5) and (sources is None or f"src{i % 3}" in sources)]
        return [f"c{i}" for i in sorted(ok, key=lambda i: -sims[i])[:10]]

    def same(got, want):  # exact search gives the exact list; HNSW at least 9 of the 10
        ids = [r.chunk.id for r in got]
        return ids == want if index == "flat" else len(set(ids) & set(want)) >= 9

    got = store.query(rag.VectorQuery(q.tolist(), 10, "t", "ws"))
    assert same(got, exact(2000, False))
    assert got[0].chunk.embedding == pytest.approx(X[int(got[0].chunk.id[1:])].tolist())
    got = store.query(rag.VectorQuery(q.tolist(), 10, "t", "ws", allowed_groups=["eng"], source_ids=["src1"]))
    assert same(got, exact(2000, True, {"src1"}))
    # writes through this object update the resident rows
    store.upsert(chunks[2000:])
    assert same(store.query(rag.VectorQuery(q.tolist(), 10, "t", "ws")), exact(3000, False))
    top = store.query(rag.VectorQuery(q.tolist(), 1, "t", "ws"))[0].chunk
    store.delete_by_doc("t", "ws", top.source_id, top.doc_id)
    after = [r.chunk.id for r in store.query(rag.VectorQuery(q.tolist(), 10, "t", "ws"))]
    assert all(cid not in after for cid in [c.id for c in chunks if c.doc_id == top.doc_id])
    # another connection's commit drops the resident copy
    other = rag.SqliteVectorStore(db)
    moved = rag.EmbeddedChunk("new", "t", "ws", "src0", "dn", 0, "new", (q * 3).tolist())
    other.upsert([moved])
    assert store.query(rag.VectorQuery(q.tolist(), 1, "t", "ws"))[0].chunk.id == "new"


def test_hnsw_graph_is_saved_and_reloaded(tmp_path):
    from kapsl_sdk_b200 import _native

    X, _ = _clustered(3000, 32, 5)
    h = _native.rag.Hnsw(32)
    h.add(X)
    h.remove(7)
    p = str(tmp_path / "g.hnsw")
    h.save(p)
    g = _native.rag.Hnsw.load(p)
    for q in X[:20]:
        a, b = h.search(q, 10, 64), g.search(q, 10, 64)
        assert np.array_equal(a[1], b[1]) and np.allclose(a[0], b[0])
    bad = tmp_path / "bad.hnsw"
    data = bytearray(open(p, "rb").read())
    data[-4:] = (10 ** 6).to_bytes(4, "little", signed=True)  # a link to a node that does not exist
    bad.write_bytes(bytes(data))
    with pytest.raises(RuntimeError):
        _native.rag.Hnsw.load(str(bad))
    bad.write_bytes(bytes(data[:100]))
    with pytest.raises(RuntimeError):
        _native.rag.Hnsw.load(str(bad))
    # the store saves a scope's graph and a later store loads it instead of rebuilding
    db, idx = str(tmp_path / "v.db"), str(tmp_path / "graphs")
    s1 = rag.SqliteVectorStore(db, index="hnsw", exact_below=10, index_dir=idx)
    s1.upsert([rag.EmbeddedChunk(f"c{i}", "t", "ws", "s", "d", i, "x", X[i].tolist()) for i in range(3000)])
    r1 = [r.chunk.id for r in s1.query(rag.VectorQuery(X[3].tolist(), 5, "t", "ws"))]
    files = os.listdir(idx)
    assert len(files) == 1
    mtime = os.path.getmtime(os.path.join(idx, files[0]))
    s2 = rag.SqliteVectorStore(db, index="hnsw", exact_below=10, index_dir=idx)
    assert [r.chunk.id for r in s2.query(rag.VectorQuery(X[3].tolist(), 5, "t", "ws"))] == r1
    assert os.listdir(idx) == files and os.path.getmtime(os.path.join(idx, files[0])) == mtime  # loaded
    s2.upsert([rag.EmbeddedChunk("new", "t", "ws", "s", "d", 0, "x", X[3].tolist())])
    assert s2.query(rag.VectorQuery(X[3].tolist(), 2, "t", "ws"))[0].chunk.id in ("new", "c3")


def test_hnsw_saved_graph_rebuilt_after_same_second_reupsert(tmp_path):
    """Re-upserting the last chunk with a new vector keeps its id, row order and
    (within one second) its update time; the saved graph must still be rebuilt."""
    X, _ = _clustered(600, 16, 4)
    db, idx = str(tmp_path / "v.db"), str(tmp_path / "graphs")
    s1 = rag.SqliteVectorStore(db, index="hnsw", exact_below=10, index_dir=idx)
    s1.upsert([rag.EmbeddedChunk(f"c{i}", "t", "ws", "s", "d", i, "x", X[i].tolist()) for i in range(600)])
    s1.query(rag.VectorQuery(X[0].tolist(), 3, "t", "ws"))  # builds and saves the graph
    saved1 = [f for f in os.listdir(idx) if f.endswith(".hnsw")]
    assert len(saved1) == 1
    far = -X[0] * 5.0
    s1.upsert([rag.EmbeddedChunk("c599", "t", "ws", "s", "d", 599, "x", far.tolist())])
    s2 = rag.SqliteVectorStore(db, index="hnsw", exact_below=10, index_dir=idx)
    assert s2.query(rag.VectorQuery(X[5].tolist(), 3, "t", "ws"))[0].chunk.id == "c5"
    # the stale graph was not loaded: a graph under the new key replaced it (the
    # search itself is approximate, so the file name is the deterministic check)
    saved2 = [f for f in os.listdir(idx) if f.endswith(".hnsw")]
    assert len(saved2) == 1 and saved2 != saved1
