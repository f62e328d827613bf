"""Tokenizers for the LLM backend.

* ``HFTokenizer``: a HuggingFace ``tokenizer.json`` through the ``tokenizers``
  library (the reference uses tokenizers 0.20.4 the same way,
  crates/kapsl-llm/Cargo.toml).
* ``GGUFTokenizer``: the tokenizer stored in GGUF metadata: SentencePiece
  BPE (score-ordered merges, ``<0xNN>`` byte fallback) or byte-level BPE
  (``tokenizer.ggml.merges`` with the named pre-tokenizer pattern).
* ``ByteTokenizer``: UTF-8 bytes as ids (offset 3, 0-2 reserved for
  pad/bos/eos) for random-init models that ship no vocabulary.
"""
from __future__ import annotations

import json
import os
from typing import Optional


class ByteTokenizer:
    OFFSET = 3

    def __init__(self, vocab_size: int = 259, bos_id: Optional[int] = 1, eos_id: Optional[int] = 2):
        self.vocab_size = max(vocab_size, 259)
        self.bos_id = bos_id
        self.eos_id = eos_id

    def encode(self, text: str, add_bos: bool = False) -> list:
        ids = [b + self.OFFSET for b in text.encode("utf-8")]
        return ([self.bos_id] if add_bos and self.bos_id is not None else []) + ids

    def decode(self, ids) -> str:
        out = bytes(i - self.OFFSET for i in ids if self.OFFSET <= i < self.OFFSET + 256)
        return out.decode("utf-8", errors="replace")


class HFTokenizer:
    def __init__(self, path: str):
        from tokenizers import Tokenizer

        self.tok = Tokenizer.from_file(path)
        with open(path) as f:
            self.json = json.load(f)
        self.vocab_size = self.tok.get_vocab_size()
        self.bos_id = None
        self.eos_id = None

    def encode(self, text: str, add_bos: bool = False) -> list:
        ids = self.tok.encode(text, add_special_tokens=False).ids
        if add_bos and self.bos_id is not None and (not ids or ids[0] != self.bos_id):
            ids = [self.bos_id] + ids
        return ids

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True)


# Byte-level BPE pre-tokenizer patterns by GGUF ``tokenizer.ggml.pre`` name
# (the split rules published with each tokenizer; `regex` syntax).
_BPE_PATTERNS = {
    "gpt2": r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+""",
    "llama-bpe": (r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*"""
                  r"""|\s*[\r\n]+|\s+(?!\S)|\s+"""),
    "qwen2": (r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*"""
              r"""|\s*[\r\n]+|\s+(?!\S)|\s+"""),
}
_BPE_PATTERNS["default"] = _BPE_PATTERNS["gpt2"]
_BPE_PATTERNS["llama3"] = _BPE_PATTERNS["llama-bpe"]


def _bytes_to_unicode() -> dict:
    """The byte -> printable character table of byte-level BPE (GPT-2)."""
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(ord("\xa1"), ord("\xac") + 1)) + \
        list(range(ord("\xae"), ord("\xff") + 1))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    return dict(zip(bs, (chr(c) for c in cs)))


class GGUFTokenizer:
    """The tokenizer stored in GGUF metadata.

    * ``model == "llama"`` (SentencePiece BPE): spaces become ``▁`` (with a
      leading one), the text is split into characters, and the adjacent pair
      whose concatenation is a vocabulary piece with the highest score is
      merged until none is left; characters outside the vocabulary fall back
      to ``<0xNN>`` byte pieces.
    * ``model == "gpt2"`` (byte-level BPE, Llama 3 / Qwen2): the text is split
      by the pre-tokenizer pattern named by ``tokenizer.ggml.pre``, each piece's
      UTF-8 bytes are mapped to printable characters, and ``tokenizer.ggml.merges``
      are applied lowest rank first.
    In both, control and user-defined tokens written in the text (chat
    template markers) are matched first and emitted as single ids."""
    SPACE = "\u2581"

    def __init__(self, tokens: list, scores: Optional[list] = None, token_types: Optional[list] = None,
                 bos_id: Optional[int] = 1, eos_id: Optional[int] = 2, model: str = "llama",
                 merges: Optional[list] = None, pre: Optional[str] = None, add_space_prefix: bool = True):
        self.tokens = list(tokens)
        self.vocab_size = len(self.tokens)
        self.scores = list(scores) if scores is not None else [0.0] * len(self.tokens)
        self.types = list(token_types) if token_types is not None else [1] * len(self.tokens)
        self.bos_id, self.eos_id = bos_id, eos_id
        self.model = model
        self.add_space_prefix = add_space_prefix
        self.index = {}
        for i, t in enumerate(self.tokens):
            self.index.setdefault(t, i)
        self.byte_ids = {}
        for i, t in enumerate(self.tokens):
            if len(t) == 6 and t.startswith("<0x") and t.endswith(">"):
                try:
                    self.byte_ids[int(t[3:5], 16)] = i
                except ValueError:
                    pass
        # control (3) and user-defined (4) tokens are matched verbatim in the text, longest first
        self.special = sorted((t for i, t in enumerate(self.tokens) if self.types[i] in (3, 4) and t),
                              key=len, reverse=True)
        if model == "gpt2":
            import regex

            if not merges:
                raise ValueError("byte-level BPE tokenizer without merges")
            self.ranks = {tuple(m.split(" ", 1)): r for r, m in enumerate(merges)}
            pat = _BPE_PATTERNS.get(pre or "default")
            if pat is None:
                raise ValueError(f"unknown BPE pre-tokenizer {pre!r}")
            self.pat = regex.compile(pat)
            self.b2u = _bytes_to_unicode()
            self.u2b = {v: k for k, v in self.b2u.items()}
        elif model != "llama":
            raise ValueError(f"GGUF tokenizer model {model!r} is not supported")

    # ------------------------------------------------------------- encode
    def _split_special(self, text: str) -> list:
        """[(is_special, piece)] with control / user-defined tokens cut out."""
        if not self.special:
            return [(False, text)]
        out, i, start = [], 0, 0
        while i < len(text):
            for t in self.special:
                if text.startswith(t, i):
                    if start < i:
                        out.append((False, text[start:i]))
                    out.append((True, t))
                    i += len(t)
                    start = i
                    break
            else:
                i += 1
        if start < len(text):
            out.append((False, text[start:]))
        return out

    def _spm(self, text: str, first: bool) -> list:
        s = text.replace(" ", self.SPACE)
        if first and self.add_space_prefix:
            s = self.SPACE + s
        sym = list(s)
        import heapq

        def pair_score(i):
            tid = self.index.get(sym[i] + sym[i + 1])
            return None if tid is None else (-self.scores[tid], i)

        # symbols live in a linked list; the heap holds candidate merges (stale ones are skipped)
        nxt = list(range(1, len(sym) + 1))
        prv = list(range(-1, len(sym) - 1))
        alive = [True] * len(sym)
        heap = []
        for i in range(len(sym) - 1):
            sc = pair_score(i)
            if sc is not None:
                heapq.heappush(heap, (sc[0], i, sym[i] + sym[i + 1]))
        while heap:
            _, i, merged = heapq.heappop(heap)
            j = nxt[i]
            if not alive[i] or j >= len(sym) or not alive[j] or sym[i] + sym[j] != merged:
                continue
            sym[i] = merged
            alive[j] = False
            nxt[i] = nxt[j]
            if nxt[j] < len(sym):
                prv[nxt[j]] = i
            for a in (prv[i], i):
                if a >= 0 and alive[a] and nxt[a] < len(sym):
                    tid = self.index.get(sym[a] + sym[nxt[a]])
                    if tid is not None:
                        heapq.heappush(heap, (-self.scores[tid], a, sym[a] + sym[nxt[a]]))
        ids = []
        i = 0
        while i < len(sym):
            if alive[i]:
                tid = self.index.get(sym[i])
                if tid is not None:
                    ids.append(tid)
                else:
                    ids.extend(self.byte_ids.get(b, 0) for b in sym[i].encode("utf-8"))
            i = nxt[i] if alive[i] else i + 1
        return ids

    def _bpe_piece(self, piece: str) -> list:
        word = [self.b2u[b] for b in piece.encode("utf-8")]
        while len(word) > 1:
            best, bi = None, -1
            for i in range(len(word) - 1):
                r = self.ranks.get((word[i], word[i + 1]))
                if r is not None and (best is None or r < best):
                    best, bi = r, i
            if best is None:
                break
            a, b = word[bi], word[bi + 1]
            out, i = [], 0
            while i < len(word):  # merge every occurrence of the pair, left to right
                if i < len(word) - 1 and word[i] == a and word[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(word[i])
                    i += 1
            word = out
        return [self.index[w] for w in word if w in self.index]

    def encode(self, text: str, add_bos: bool = False) -> list:
        ids = []
        first = True
        for special, piece in self._split_special(text):
            if special:
                ids.append(self.index[piece])
            elif self.model == "gpt2":
                for m in self.pat.findall(piece):
                    ids.extend(self._bpe_piece(m))
            else:
                ids.extend(self._spm(piece, first))
            first = False
        return ([self.bos_id] if add_bos and self.bos_id is not None else []) + ids

    # ------------------------------------------------------------- decode
    def decode(self, ids) -> str:
        parts = bytearray()
        for i in ids:
            if i < 0 or i >= self.vocab_size:
                continue
            t = self.tokens[i]
            if self.types[i] in (2, 3):  # unknown / control
                continue
            if self.model == "gpt2":
                parts.extend(bytes(self.u2b[c] for c in t if c in self.u2b))
                continue
            if self.types[i] == 6 or (len(t) == 6 and t.startswith("<0x") and t.endswith(">")):
                try:
                    parts.append(int(t[3:5], 16))
                    continue
                except ValueError:
                    pass
            parts.extend(t.encode("utf-8"))
        out = parts.decode("utf-8", errors="replace")
        if self.model == "gpt2":
            return out
        out = out.replace(self.SPACE, " ")
        return out[1:] if out.startswith(" ") and self.add_space_prefix else out


def load_tokenizer(model_dir: Optional[str], vocab_size: int, bos_id=None, eos_id=None):
    if model_dir:
        p = os.path.join(model_dir, "tokenizer.json")
        if os.path.isfile(p):
            t = HFTokenizer(p)
            t.bos_id, t.eos_id = bos_id, eos_id
            return t
    return ByteTokenizer(vocab_size, bos_id if bos_id is not None else 1, eos_id if eos_id is not None else 2)
