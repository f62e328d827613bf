"""GGUF tokenizers against their reference implementations: SentencePiece
BPE (a model trained here with the sentencepiece library) and byte-level BPE
(the same vocabulary and merges loaded into the HuggingFace tokenizers
library with the GPT-2 / Llama 3 pre-tokenizers)."""
import json
import os

import pytest

from kapsl_sdk_b200.llm.tokenizer import GGUFTokenizer

TEXTS = ["Hello world", "The quick brown fox jumps over the lazy dog.", "  leading and  double  spaces",
         "numbers 12345 and 3.14159", "ünïcödé — text ✓ with 中文 characters", "tabs\tand\nnewlines\n\nhere",
         "it's we're they'll I'd", ""]

CORPUS = ("the quick brown fox jumps over the lazy dog " * 3 + "hello world hello there general kenobi "
          "tokenizers split words into pieces and pieces into tokens numbers 123 456 7890 ") * 20


def test_sentencepiece_bpe_matches_sentencepiece(tmp_path):
    spm = pytest.importorskip("sentencepiece")
    corpus = tmp_path / "c.txt"
    words = CORPUS.split()
    corpus.write_text("\n".join(" ".join(words[i:i + 12]) for i in range(0, len(words), 12)) + "\nünïcödé ✓ 中文\n")
    prefix = str(tmp_path / "m")
    spm.SentencePieceTrainer.train(input=str(corpus), model_prefix=prefix, vocab_size=400, model_type="bpe",
                                   byte_fallback=True, character_coverage=1.0, bos_id=1, eos_id=2, unk_id=0,
                                   pad_id=-1, minloglevel=2, normalization_rule_name="identity",
                                   remove_extra_whitespaces=False)  # as the Llama tokenizer
    sp = spm.SentencePieceProcessor(model_file=prefix + ".model")
    tokens = [sp.id_to_piece(i) for i in range(sp.get_piece_size())]
    scores = [sp.get_score(i) for i in range(sp.get_piece_size())]
    types = [2 if sp.is_unknown(i) else 3 if sp.is_control(i) else 6 if sp.is_byte(i) else 1
             for i in range(sp.get_piece_size())]
    tok = GGUFTokenizer(tokens, scores, types, bos_id=1, eos_id=2, model="llama")
    for t in TEXTS + ["the quick brown", "hello kenobi 999"]:
        assert tok.encode(t) == sp.encode(t), t
        assert tok.decode(tok.encode(t)) == sp.decode(sp.encode(t)), t


@pytest.mark.parametrize("pre", ["gpt2", "llama-bpe", "qwen2"])
def test_byte_level_bpe_matches_hf_tokenizers(tmp_path, pre):
    from tokenizers import Regex, Tokenizer, decoders, models, pre_tokenizers, trainers

    from kapsl_sdk_b200.llm.tokenizer import _BPE_PATTERNS

    t = Tokenizer(models.BPE())
    t.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(_BPE_PATTERNS[pre]), behavior="isolated"),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    t.decoder = decoders.ByteLevel()
    t.train_from_iterator([CORPUS] * 5, trainers.BpeTrainer(vocab_size=400, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                                            special_tokens=["<|begin|>", "<|end|>"]))
    path = tmp_path / "tok.json"
    t.save(str(path))
    data = json.loads(path.read_text())
    vocab = data["model"]["vocab"]
    merges = [m if isinstance(m, str) else " ".join(m) for m in data["model"]["merges"]]
    tokens = [None] * len(vocab)
    for s, i in vocab.items():
        tokens[i] = s
    types = [3 if s in ("<|begin|>", "<|end|>") else 1 for s in tokens]
    tok = GGUFTokenizer(tokens, None, types, bos_id=vocab["<|begin|>"], eos_id=vocab["<|end|>"], model="gpt2",
                        merges=merges, pre=pre)
    for text in TEXTS:
        assert tok.encode(text) == t.encode(text).ids, text
        assert tok.decode(tok.encode(text)) == text
    both = "<|begin|>hello world<|end|>"
    ids = tok.encode(both)
    assert ids[0] == vocab["<|begin|>"] and ids[-1] == vocab["<|end|>"]
    assert ids[1:-1] == t.encode("hello world").ids
