"""Tokenizers for the LLM backend.

* ``HFTokenizer``: a HuggingFace ``tokenizer.json`` through the ``tokenizers``
  library (the reference uses tokenizers 0.20.4 the same way,
  crates/kapsl-llm/Cargo.toml).
* ``GGUFTokenizer``: the vocabulary stored in GGUF metadata
  (``tokenizer.ggml.tokens`` / ``scores`` / ``token_type``), greedy longest
  match over SentencePiece-style pieces (``▁`` for spaces, ``<0xNN>`` byte
  fallback) -- enough for the GGUF path without external files.
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


class GGUFTokenizer:
    SPACE = "▁"

    def __init__(self, tokens: list, scores: Optional[list] = None, token_types: Optional[list] = None,
                 bos_id: Optional[int] = 1, eos_id: Optional[int] = 2):
        self.tokens = list(tokens)
        self.vocab_size = len(self.tokens)
        self.types = list(token_types) if token_types is not None else [1] * len(self.tokens)
        self.bos_id, self.eos_id = bos_id, eos_id
        self.index = {}
        for i, t in enumerate(self.tokens):
            if self.types[i] in (1, 4, 6):  # normal, user-defined, byte
                self.index.setdefault(t, i)
        self.max_len = max((len(t) for t in self.index), default=1)
        self.byte_ids = {}
        for i, t in enumerate(self.tokens):
            if len(t) == 6 and t.startswith("<0x") and t.endswith(">"):
                try:
                    self.byte_ids[int(t[3:5], 16)] = i
                except ValueError:
                    pass

    def encode(self, text: str, add_bos: bool = False) -> list:
        s = self.SPACE + text.replace(" ", self.SPACE) if text else ""
        ids, i = [], 0
        while i < len(s):
            for n in range(min(self.max_len, len(s) - i), 0, -1):
                tid = self.index.get(s[i:i + n])
                if tid is not None:
                    ids.append(tid)
                    i += n
                    break
            else:
                for b in s[i].encode("utf-8"):
                    ids.append(self.byte_ids.get(b, 0))
                i += 1
        return ([self.bos_id] if add_bos and self.bos_id is not None else []) + ids

    def decode(self, ids) -> str:
        parts = bytearray()
        for i in ids:
            if i < 0 or i >= self.vocab_size:
                continue
            t = self.tokens[i]
            if self.types[i] == 6 or (len(t) == 6 and t.startswith("<0x") and t.endswith(">")):
                try:
                    parts.append(int(t[3:5], 16))
                    continue
                except ValueError:
                    pass
            if self.types[i] in (2, 3):  # unknown / control
                continue
            parts.extend(t.encode("utf-8"))
        out = parts.decode("utf-8", errors="replace").replace(self.SPACE, " ")
        return out[1:] if out.startswith(" ") else out


def load_tokenizer(model_dir: Optional[str], vocab_size: int, bos_id=None, eos_id=None):
    if model_dir:
        p = os.path.join(model_dir, "tokenizer.json")
        if os.path.isfile(p):
            t = HFTokenizer(p)
            t.bos_id, t.eos_id = bos_id, eos_id
            return t
    return ByteTokenizer(vocab_size, bos_id if bos_id is not None else 1, eos_id if eos_id is not None else 2)
