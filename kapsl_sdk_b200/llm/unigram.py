"""Unigram (SentencePiece-style) tokenizer and its trainer.

The reference gets Unigram training from HF ``tokenizers``, whose trainer
takes its seed pieces from the patched esaxx-rs suffix array
(``patches/esaxx-rs/src/lib.rs:110-215``, ``esaxx.cpp:623``).  Here the same
capability is native: ``_native.text`` builds the suffix array (SA-IS), the
LCP array and the suffix tree's internal nodes (every substring that repeats,
with its count), and runs the Unigram lattice (Viterbi and forward-backward
expected counts) in C++ over a code-point trie.

Training follows Kudo, "Subword Regularization" (ACL 2018):

1. Sentences are normalised (spaces -> ``▁``, a leading ``▁``) and split into
   words that start at a ``▁``; word counts weight everything below.
2. Seed pieces: every character, plus the repeated substrings of the corpus
   (up to ``max_piece_len`` code points, ``▁`` only in front) with the largest
   ``occurrences * length``, at most ``seed_size`` of them.
3. EM: expected piece counts over every word's lattice, then
   ``log p = log(count / total)``; pieces whose expected count drops below
   0.5 are removed (characters never are).
4. Pruning: a piece's loss is ``count * (log p(piece) - sum log p(alt))``
   where ``alt`` is its best segmentation without it; the pieces with the
   smallest loss go, ``shrinking_factor`` of the vocabulary kept per round,
   until ``vocab_size`` is reached.

Meta pieces ``<unk>``, ``<s>``, ``</s>`` take ids 0-2 (SentencePiece's
order), then, with ``byte_fallback``, the 256 ``<0xNN>`` pieces; learned
pieces follow in descending score.
"""
from __future__ import annotations

import json
import math
import re
from collections import Counter
from typing import Iterable, Optional

SPACE = "▁"
_WORD = re.compile(SPACE + "[^" + SPACE + "]*|[^" + SPACE + "]+")


def _text():
    from .. import _native

    return _native.text


def normalize(text: str, add_dummy_prefix: bool = True) -> str:
    t = text.replace(" ", SPACE)
    if add_dummy_prefix and t and not t.startswith(SPACE):
        t = SPACE + t
    return t


def split_words(normalized: str) -> list:
    return _WORD.findall(normalized)


def suffix_array(text: str) -> list:
    """Start offsets of the suffixes of ``text`` (code points) in sorted order."""
    return list(_text().suffix_array(text))


def repeated_substrings(text: str) -> list:
    """[(substring, occurrences)] for every internal node of the suffix tree of
    ``text``, bottom-up, the root ``("", len(text))`` last: the substrings that
    occur at least twice and are followed by two different characters (or by
    the end of the text)."""
    return list(_text().repeated_substrings(text))


class UnigramTokenizer:
    """Viterbi segmentation over scored pieces.  Characters that no piece covers
    become ``<unk>``, or their UTF-8 bytes ``<0xNN>`` with ``byte_fallback``."""

    def __init__(self, pieces: list, scores: list, unk_id: int = 0, bos_id: Optional[int] = 1,
                 eos_id: Optional[int] = 2, add_dummy_prefix: bool = True, byte_fallback: bool = False):
        if len(pieces) != len(scores):
            raise ValueError("pieces and scores differ in length")
        self.pieces, self.scores = list(pieces), [float(s) for s in scores]
        self.vocab_size = len(self.pieces)
        self.unk_id, self.bos_id, self.eos_id = unk_id, bos_id, eos_id
        self.add_dummy_prefix, self.byte_fallback = add_dummy_prefix, byte_fallback
        self.index = {}
        for i, p in enumerate(self.pieces):
            self.index.setdefault(p, i)
        self.byte_ids = {}
        for i, p in enumerate(self.pieces):
            if len(p) == 6 and p.startswith("<0x") and p.endswith(">"):
                self.byte_ids[int(p[3:5], 16)] = i
        self.id_to_byte = {v: k for k, v in self.byte_ids.items()}
        if byte_fallback and len(self.byte_ids) < 256:
            raise ValueError("byte_fallback needs the 256 <0xNN> pieces")
        meta = {unk_id, bos_id, eos_id} | set(self.byte_ids.values())
        # meta and byte pieces never match text; unk is the lattice's fallback edge
        lattice = [("" if i in meta else p) for i, p in enumerate(self.pieces)]
        self._model = _text().UnigramModel(lattice, self.scores, unk_id if unk_id is not None else -1)
        self._cache: dict = {}

    def _word(self, w: str) -> list:
        ids = self._cache.get(w)
        if ids is None:
            ids = list(self._model.encode(w))
            if self.byte_fallback and self.unk_id in ids:
                ids = self._bytes_for_unk(w, ids)
            if len(self._cache) < 65536:
                self._cache[w] = ids
        return ids

    def _bytes_for_unk(self, w: str, ids: list) -> list:
        out, pos = [], 0
        for i in ids:
            if i == self.unk_id:
                out.extend(self.byte_ids[b] for b in w[pos].encode("utf-8"))
                pos += 1
            else:
                out.append(i)
                pos += len(self.pieces[i])
        return out

    def encode(self, text: str, add_bos: bool = False) -> list:
        ids = [self.bos_id] if add_bos and self.bos_id is not None else []
        for w in split_words(normalize(text, self.add_dummy_prefix)):
            ids.extend(self._word(w))
        return ids

    def decode(self, ids) -> str:
        out, pending = [], bytearray()
        for i in ids:
            i = int(i)
            if i in (self.bos_id, self.eos_id):
                continue
            b = self.id_to_byte.get(i)
            if b is not None:
                pending.append(b)
                continue
            if pending:
                out.append(pending.decode("utf-8", errors="replace"))
                pending = bytearray()
            out.append(" ⁇ " if i == self.unk_id else self.pieces[i])
        if pending:
            out.append(pending.decode("utf-8", errors="replace"))
        s = "".join(out).replace(SPACE, " ")
        return s[1:] if self.add_dummy_prefix and s.startswith(" ") else s

    # ------------------------------------------------------------ persistence
    def to_hf_json(self) -> dict:
        """A ``tokenizer.json`` for HF ``tokenizers`` (Metaspace pre-tokenizer,
        Unigram model) that segments text the same way."""
        return {
            "version": "1.0", "truncation": None, "padding": None, "added_tokens": [], "normalizer": None,
            "pre_tokenizer": {"type": "Metaspace", "replacement": SPACE,
                              "prepend_scheme": "always" if self.add_dummy_prefix else "never", "split": True},
            "post_processor": None,
            "decoder": {"type": "Metaspace", "replacement": SPACE,
                        "prepend_scheme": "always" if self.add_dummy_prefix else "never", "split": True},
            "model": {"type": "Unigram", "unk_id": self.unk_id, "byte_fallback": self.byte_fallback,
                      "vocab": [[p, s] for p, s in zip(self.pieces, self.scores)]},
        }

    def save(self, path: str) -> None:
        with open(path, "w", encoding="utf-8") as f:
            json.dump(self.to_hf_json(), f, ensure_ascii=False)

    @classmethod
    def load(cls, path: str, bos_id: Optional[int] = 1, eos_id: Optional[int] = 2) -> "UnigramTokenizer":
        with open(path, encoding="utf-8") as f:
            j = json.load(f)
        m = j["model"]
        if m.get("type") != "Unigram":
            raise ValueError(f"{path}: not a Unigram model")
        pre = j.get("pre_tokenizer") or {}
        return cls([p for p, _ in m["vocab"]], [s for _, s in m["vocab"]], unk_id=m.get("unk_id", 0),
                   bos_id=bos_id, eos_id=eos_id, add_dummy_prefix=pre.get("prepend_scheme", "always") != "never",
                   byte_fallback=bool(m.get("byte_fallback", False)))


# -------------------------------------------------------------------- trainer
def _seed_pieces(sentences: list, chars: Counter, max_piece_len: int, seed_size: int,
                 max_corpus_chars: int) -> dict:
    buf, total = [], 0
    for s in sentences:
        if total + len(s) + 1 > max_corpus_chars:
            break
        buf.append(s)
        total += len(s) + 1
    corpus = "\0".join(buf)
    cand = _text().top_repeated_substrings(corpus, max_piece_len, seed_size, "\0", SPACE)
    seeds = {c: float(f) for c, f in chars.items()}
    for sub, freq in cand:
        seeds[sub] = float(freq * len(sub))
    total = sum(seeds.values())
    return {p: math.log(v) - math.log(total) for p, v in seeds.items()}


def _em(pieces: list, scores: list, words: list, freqs: list, required: set):
    model = _text().UnigramModel(pieces, scores, -1)
    counts, loglik = model.expected_counts(words, freqs)
    keep = [i for i, c in enumerate(counts) if c >= 0.5 or pieces[i] in required]
    kept_counts = [max(counts[i], 0.5) for i in keep]
    total = sum(kept_counts)
    return [pieces[i] for i in keep], [math.log(c) - math.log(total) for c in kept_counts], kept_counts, loglik


def train_unigram(sentences: Iterable[str], vocab_size: int, *, max_piece_len: int = 16, seed_size: int = 200_000,
                  shrinking_factor: float = 0.75, em_iters: int = 2, add_dummy_prefix: bool = True,
                  byte_fallback: bool = False, max_corpus_chars: int = 50_000_000,
                  history: Optional[list] = None) -> UnigramTokenizer:
    """Train a Unigram tokenizer of ``vocab_size`` pieces (meta and byte pieces
    included).  ``history``, when given, receives the corpus log-likelihood
    after every EM step."""
    norm = [normalize(s, add_dummy_prefix) for s in sentences if s]
    wc = Counter()
    for s in norm:
        wc.update(split_words(s))
    words, freqs = list(wc.keys()), [float(v) for v in wc.values()]
    chars = Counter()
    for w, f in wc.items():
        for c in w:
            chars[c] += f
    required = set(chars)
    meta = ["<unk>", "<s>", "</s>"] + ([f"<0x{b:02X}>" for b in range(256)] if byte_fallback else [])
    target = vocab_size - len(meta)
    if target < len(required):
        raise ValueError(f"vocab_size {vocab_size} is below the {len(required)} characters plus {len(meta)} meta pieces")
    seeds = _seed_pieces(norm, chars, max_piece_len, seed_size, max_corpus_chars)
    pieces, scores = list(seeds.keys()), list(seeds.values())
    for _ in range(1000):
        for _ in range(em_iters):
            pieces, scores, counts, ll = _em(pieces, scores, words, freqs, required)
            if history is not None:
                history.append(ll)
        if len(pieces) <= target:
            break
        alt = _text().UnigramModel(pieces, scores, -1).alternative_scores()
        loss = [(counts[i] * (scores[i] - max(alt[i], -1e9)), i) for i, p in enumerate(pieces) if p not in required]
        loss.sort(reverse=True)
        size = max(target, int(len(pieces) * shrinking_factor))
        keep = {i for i, p in enumerate(pieces) if p in required}
        keep.update(i for _, i in loss[:max(0, size - len(keep))])
        pieces = [p for i, p in enumerate(pieces) if i in keep]
        scores = [s for i, s in enumerate(scores) if i in keep]
    order = sorted(range(len(pieces)), key=lambda i: (-scores[i], pieces[i]))
    if len(order) > target:  # the last EM kept more than asked: drop the lowest non-characters
        drop = [i for i in reversed(order) if pieces[i] not in required][:len(order) - target]
        order = [i for i in order if i not in set(drop)]
    floor = min(scores) if scores else 0.0
    all_pieces = meta + [pieces[i] for i in order]
    all_scores = [0.0] * 3 + [floor - 1.0] * (len(meta) - 3) + [scores[i] for i in order]
    return UnigramTokenizer(all_pieces, all_scores, unk_id=0, bos_id=1, eos_id=2,
                            add_dummy_prefix=add_dummy_prefix, byte_fallback=byte_fallback)


def main(argv: Optional[list] = None) -> int:
    """``python -m kapsl_sdk_b200.llm.unigram corpus.txt [more.txt ...] --vocab-size 8000 -o tokenizer.json``:
    train on the lines of the given files and write an HF ``tokenizer.json``."""
    import argparse

    p = argparse.ArgumentParser(prog="python -m kapsl_sdk_b200.llm.unigram", description=main.__doc__)
    p.add_argument("files", nargs="+")
    p.add_argument("--vocab-size", type=int, default=8000)
    p.add_argument("--max-piece-len", type=int, default=16)
    p.add_argument("--byte-fallback", action="store_true")
    p.add_argument("-o", "--output", default="tokenizer.json")
    a = p.parse_args(argv)
    lines = []
    for f in a.files:
        with open(f, encoding="utf-8", errors="replace") as fh:
            lines.extend(line.rstrip("\n") for line in fh if line.strip())
    tok = train_unigram(lines, a.vocab_size, max_piece_len=a.max_piece_len, byte_fallback=a.byte_fallback)
    tok.save(a.output)
    n_tok = sum(len(tok.encode(s)) for s in lines[:10000])
    n_chr = sum(len(s) for s in lines[:10000])
    print(f"{a.output}: {tok.vocab_size} pieces, {n_chr / max(n_tok, 1):.2f} characters per token")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
