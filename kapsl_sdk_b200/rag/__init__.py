"""Retrieval-augmented generation: connector protocol and runtimes, ingestion,
document and vector stores, prompt assembly (reference crates kapsl-rag and
kapsl-rag-sdk, and crates/kapsl-llm/src/rag.rs)."""
from .ingestion import (Chunk, DummyEmbedder, HashEmbedder, IngestionContext, IngestionPipeline, ModelEmbedder,
                        ParsedDocument, PlainTextParser, SimpleChunker)
from .prompt import Citation, RagChunk, RagPrompt, RagPromptConfig, build_rag_prompt, select_chunks
from .protocol import (ConnectorManifest, ConnectorRemoteError, DocumentDelta, DocumentPayload, ExternalAcl,
                       SourceDescriptor)
from .runtime import ConnectorClient, ExtensionManager, ExtensionRegistry, SidecarRuntime, WasmRuntime
from .server import Connector, ConnectorError, serve_stdio
from .store import AccessControl, DocKey, EmbeddedChunk, FsDocStore, SqliteVectorStore, VectorQuery
