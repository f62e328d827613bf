"""Suffix array / repeated substrings (the esaxx capability) and the Unigram
tokenizer and trainer built on them; oracles are brute force and HF
``tokenizers``."""
import json
import math
import os
import random
from collections import Counter

import pytest

from kapsl_sdk_b200.llm import unigram as U

WORDS = ["the", "quick", "brown", "fox", "jumps", "over", "lazy", "dog", "tokenizer", "training", "unigram",
         "model", "language", "piece", "sentence", "subword", "regularization", "über", "naïve", "日本語"]


def corpus(n=1500, seed=0):
    r = random.Random(seed)
    return [" ".join(r.choice(WORDS) + r.choice(["", "s", "ed", "ing"]) for _ in range(r.randint(3, 14)))
            for _ in range(n)]


def test_suffix_and_lcp_arrays_match_brute_force():
    from kapsl_sdk_b200 import _native

    r = random.Random(1)
    for _ in range(1500):
        alpha = r.choice(["ab", "abc", "a", "abcdefgh", "é▁x日"])
        s = "".join(r.choice(alpha) for _ in range(r.randint(0, 60)))
        sa = sorted(range(len(s)), key=lambda i: s[i:])
        assert U.suffix_array(s) == sa
        lcp = [0] * min(1, len(s)) + [len(os.path.commonprefix([s[sa[i - 1]:], s[sa[i]:]])) for i in range(1, len(s))]
        assert list(_native.text.lcp_array(s)) == lcp


def test_repeated_substrings_match_esaxx_semantics():
    # the documented example of the reference's esaxx-rs `suffix()` iterator
    assert U.repeated_substrings("abracadabra") == [("abra", 2), ("a", 5), ("bra", 2), ("ra", 2), ("", 11)]
    r = random.Random(2)
    for _ in range(400):
        s = "".join(r.choice("abc") for _ in range(r.randint(1, 30)))
        # brute force: substrings seen twice or more whose following characters
        # (the end of the text counting as one) are not all the same
        expect = Counter({("", len(s)): 1})  # the root: every suffix
        for n in range(1, len(s)):
            subs = {s[i:i + n] for i in range(len(s) - n + 1)}
            for u in subs:
                starts = [i for i in range(len(s) - n + 1) if s.startswith(u, i)]
                nxt = {s[i + n] if i + n < len(s) else None for i in starts}
                if len(starts) >= 2 and len(nxt) >= 2:
                    expect[(u, len(starts))] += 1
        got = U.repeated_substrings(s)
        assert got[-1] == ("", len(s))
        assert Counter(got) == expect, s


def _all_segmentations(t, pieces):
    if not t:
        yield []
        return
    for j in range(1, len(t) + 1):
        if t[:j] in pieces:
            for rest in _all_segmentations(t[j:], pieces):
                yield [t[:j]] + rest


def test_lattice_viterbi_and_expected_counts_match_enumeration():
    from kapsl_sdk_b200 import _native

    r = random.Random(3)
    for _ in range(60):
        chars = "abc"
        pieces = list(chars) + sorted({"".join(r.choice(chars) for _ in range(r.randint(2, 4))) for _ in range(8)})
        scores = [r.uniform(-6, -0.5) for _ in pieces]
        sc = dict(zip(pieces, scores))
        m = _native.text.UnigramModel(pieces, scores, -1)
        words = ["".join(r.choice(chars) for _ in range(r.randint(1, 9))) for _ in range(5)]
        freqs = [float(r.randint(1, 4)) for _ in words]
        exp = [0.0] * len(pieces)
        ll = 0.0
        for w, f in zip(words, freqs):
            segs = list(_all_segmentations(w, set(pieces)))
            lps = [sum(sc[p] for p in seg) for seg in segs]
            best = segs[max(range(len(segs)), key=lambda i: lps[i])]
            assert [pieces[i] for i in m.encode(w)] == best
            z = math.log(sum(math.exp(v) for v in lps))
            ll += f * z
            for seg, lp in zip(segs, lps):
                for p in seg:
                    exp[pieces.index(p)] += f * math.exp(lp - z)
        counts, got_ll = m.expected_counts(words, freqs)
        assert got_ll == pytest.approx(ll, rel=1e-9)
        assert counts == pytest.approx(exp, rel=1e-9, abs=1e-12)
        for i, p in enumerate(pieces):  # best segmentation without the piece itself
            alt = [pieces[a] for a in m.alternative(i)]
            if len(p) == 1:
                assert alt == []
            else:
                segs = [s for s in _all_segmentations(p, set(pieces) - {p})]
                assert alt == max(segs, key=lambda s: sum(sc[x] for x in s))


def test_encoding_matches_hf_unigram_with_the_same_vocabulary():
    tokenizers = pytest.importorskip("tokenizers")
    tok = U.train_unigram(corpus(), 160)
    hf = tokenizers.Tokenizer.from_str(json.dumps(tok.to_hf_json()))
    for s in corpus(300, seed=9) + ["naïve über-models", "日本語 the fox", "unseen ß ¿ chars"]:
        assert tok.encode(s) == hf.encode(s).ids, s


def test_trainer_vocabulary_round_trip_and_likelihood():
    hist = []
    data = corpus()
    tok = U.train_unigram(data, 120, history=hist)
    assert tok.vocab_size <= 120 and tok.pieces[:3] == ["<unk>", "<s>", "</s>"]
    chars = {c for s in data for c in U.normalize(s)}
    assert chars <= set(tok.pieces)  # every character stays a piece
    assert all(p == "▁" or U.SPACE not in p[1:] for p in tok.pieces[3:])
    for s in data[:200]:
        assert tok.decode(tok.encode(s)) == s
    assert tok.encode("the fox", add_bos=True)[0] == tok.bos_id
    # EM never lowers the likelihood within one vocabulary: the last two steps share one
    assert hist[-1] >= hist[-2] - 1e-6 * abs(hist[-2])
    # compression at least as good as HF's Unigram trainer at the same vocabulary size
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers import decoders, models, pre_tokenizers, trainers

    hf = tokenizers.Tokenizer(models.Unigram())
    hf.pre_tokenizer = pre_tokenizers.Metaspace()
    hf.decoder = decoders.Metaspace()
    hf.train_from_iterator(data, trainers.UnigramTrainer(vocab_size=120, special_tokens=["<unk>"], unk_token="<unk>"))
    ours = sum(len(tok.encode(s)) for s in data)
    theirs = sum(len(hf.encode(s).ids) for s in data)
    assert ours <= theirs * 1.05, (ours, theirs)


def test_byte_fallback_and_persistence(tmp_path):
    tok = U.train_unigram(corpus(400), 400, byte_fallback=True)
    s = "the fox ¿ß"  # characters that the training text never had
    ids = tok.encode(s)
    assert tok.unk_id not in ids and tok.decode(ids) == s
    p = tmp_path / "tokenizer.json"
    tok.save(str(p))
    again = U.UnigramTokenizer.load(str(p))
    assert again.encode(s) == ids and again.pieces == tok.pieces
    plain = U.train_unigram(corpus(400), 120)
    assert plain.unk_id in plain.encode("¿") and plain.decode(plain.encode("a ¿")) .endswith("⁇ ")
    with pytest.raises(ValueError):
        U.train_unigram(["abcdefghij"], 5)


def test_command_line_trainer(tmp_path):
    src = tmp_path / "corpus.txt"
    src.write_text("\n".join(corpus(300)), encoding="utf-8")
    out = tmp_path / "tok.json"
    assert U.main([str(src), "--vocab-size", "150", "-o", str(out)]) == 0
    tok = U.UnigramTokenizer.load(str(out))
    assert tok.vocab_size <= 150 and tok.decode(tok.encode("the lazy fox")) == "the lazy fox"
