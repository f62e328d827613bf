"""Retrieval-augmented prompt assembly.

Selection: drop chunks below ``min_score``; order by score (descending, then
chunk id); optionally skip chunks whose whitespace-normalised, lower-cased
text was already taken; take at most ``max_per_source`` per source (source =
first of the metadata keys source, doc_id, document_id, file, url; else
"unknown") and ``max_chunks`` overall.  Assembly: each chunk's trimmed text,
truncated to the remaining ``max_context_tokens`` (whitespace tokens) when
``truncate`` (otherwise skipped), formatted as ``[n] text`` (bracketed) or
``text (n)`` (inline) with an optional ``Source: title | source | url`` line;
blocks joined by a blank line; citations numbered from 1.  No chunk selected:
empty context and the fallback message.

The selection and formatting rules match the reference so prompts (and the
model's citations) come out the same (crates/kapsl-llm/src/rag.rs:9-296).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Optional

SOURCE_KEYS = ("source", "doc_id", "document_id", "file", "url")


@dataclass
class RagChunk:
    id: str
    text: str
    score: float
    metadata: dict = field(default_factory=dict)


@dataclass
class RagPromptConfig:
    max_context_tokens: int = 1024
    max_chunks: int = 8
    max_per_source: int = 2
    min_score: float = 0.0
    dedupe: bool = True
    truncate: bool = True
    citation_style: str = "bracketed"  # or "inline"
    fallback_message: str = "No relevant documents found."


@dataclass
class Citation:
    index: int
    chunk_id: str
    source: Optional[str] = None
    title: Optional[str] = None
    url: Optional[str] = None


@dataclass
class RagPrompt:
    context: str
    citations: list
    used_chunks: list
    total_context_tokens: int
    truncated: bool
    fallback_message: Optional[str] = None


def whitespace_tokens(text: str) -> int:
    return len(text.split())


def _source(meta: dict) -> Optional[str]:
    for k in SOURCE_KEYS:
        if k in meta:
            return meta[k]
    return None


def _normalize(text: str) -> str:
    return " ".join(t.lower() for t in text.split())


def select_chunks(chunks: list, cfg: RagPromptConfig) -> list:
    scored = sorted((c for c in chunks if c.score >= cfg.min_score), key=lambda c: (-c.score, c.id))
    out, seen, per_source = [], set(), {}
    for c in scored:
        if len(out) >= cfg.max_chunks:
            break
        if cfg.dedupe:
            key = _normalize(c.text)
            if key in seen:
                continue
            seen.add(key)
        if cfg.max_per_source > 0:
            src = _source(c.metadata) or "unknown"
            if per_source.get(src, 0) >= cfg.max_per_source:
                continue
            per_source[src] = per_source.get(src, 0) + 1
        out.append(c)
    return out


def _source_line(c: RagChunk) -> Optional[str]:
    parts = []
    title, url, src = c.metadata.get("title"), c.metadata.get("url"), _source(c.metadata)
    if title is not None:
        parts.append(title)
    if src is not None and src not in parts:
        parts.append(src)
    if url is not None:
        parts.append(url)
    return "Source: " + " | ".join(parts) if parts else None


def build_rag_prompt(chunks: list, cfg: Optional[RagPromptConfig] = None,
                     count_tokens: Callable[[str], int] = whitespace_tokens) -> RagPrompt:
    cfg = cfg or RagPromptConfig()
    selected = select_chunks(chunks, cfg)
    if not selected:
        return RagPrompt("", [], [], 0, False, cfg.fallback_message)
    blocks, cites, used = [], [], []
    used_tokens, truncated = 0, False
    for c in selected:
        if len(blocks) >= cfg.max_chunks:
            break
        text = c.text.strip()
        if not text:
            continue
        remaining = max(0, cfg.max_context_tokens - used_tokens)
        if remaining == 0:
            break
        if count_tokens(text) > remaining:
            if not cfg.truncate:
                continue
            text = " ".join(text.split()[:remaining])
            if not text:
                break
            truncated = True
        n = len(cites) + 1
        line = _source_line(c)
        body = f"[{n}] {text}" if cfg.citation_style == "bracketed" else f"{text} ({n})"
        blocks.append(f"{body}\n{line}" if line else body)
        used_tokens += count_tokens(text)
        used.append(c)
        cites.append(Citation(n, c.id, _source(c.metadata), c.metadata.get("title"), c.metadata.get("url")))
    return RagPrompt("\n\n".join(blocks), cites, used, used_tokens, truncated, None)
