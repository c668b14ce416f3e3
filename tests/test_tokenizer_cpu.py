"""The GPT-2 byte-level BPE tokenizer (tokenizer.h; the reference's
src/tokenizer/tokenizer.cc), on CPU.

* The reference's own tests restated (tokenizer_test.cc): byte-level decode,
  BPE encode and round trip, no vocabulary / no file.
* The pre-split against the reference's pattern run by the `regex` module
  (oracle/tokenizer.py) on seeded random text: letters and numbers of many
  scripts, punctuation, emoji, every kind of whitespace, contractions,
  including the text the reference's search skips.
* Encode against the oracle's rescanning merge loop with a vocabulary and
  merges trained by the HF `tokenizers` BPE trainer on seeded text, and
  against HF's own encoder where both pre-splits agree (single spaces).
* Decode of arbitrary vocabulary strings against the reference's byte rules.
The real OLMoE vocabulary is not available offline; trained ones stand in.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

import nuthatch_b200 as nh
from oracle.tokenizer import OracleTokenizer, split

WORDS = ["the", "quick", "brown", "fox", "jumps", "over", "lazy", "dog", "Paris", "naïve", "café", "Straße",
         "東京", "数据", "Москва", "λόγος", "مرحبا", "हिन्दी", "2024", "3.14", "٣٤", "Ⅻ", "½", "don't", "it's",
         "we're", "I've", "I'm", "you'll", "he'd", "'S", "''", "!!", "?", "...", "(x)", "#1", "😀", "👍🏽", "€5"]
SPACES = [" ", "  ", "\n", "\n\n", "\t", " \n", "\r\n", " ", " ", "　", "\x0b", "\x0c", "\u0085",
          "\x1c", " \t "]


def _text(rng, n_words: int, spaces=SPACES) -> str:
    parts = []
    for _ in range(n_words):
        parts.append(WORDS[rng.integers(len(WORDS))])
        parts.append(spaces[rng.integers(len(spaces))])
    if rng.integers(2):
        parts.pop()
    return "".join(parts)


@pytest.fixture(scope="module")
def trained():
    """A byte-level BPE vocabulary and merges trained on seeded text."""
    from tokenizers import Tokenizer, models, pre_tokenizers, trainers

    rng = np.random.default_rng(3)
    corpus = [_text(rng, 40) for _ in range(300)]
    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=True)
    tr = trainers.BpeTrainer(vocab_size=1500, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                             show_progress=False)
    tok.train_from_iterator(corpus, tr)
    model = json.loads(tok.to_str())["model"]
    vocab = [t for t, _ in sorted(model["vocab"].items(), key=lambda kv: kv[1])]
    merges = [m if isinstance(m, str) else " ".join(m) for m in model["merges"]]
    return tok, vocab, merges


# ------------------------------------------------------------------ the reference's tests
def _write_gguf(path, tokens=None, merges=None, other=None):
    import gguf

    w = gguf.GGUFWriter(str(path), "olmoe")
    if tokens is not None:
        w.add_token_list(tokens)
    if merges is not None:
        w.add_token_merges(merges)
    if other is not None:
        w.add_uint32("some.key", other)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def test_decodes_byte_level(tmp_path):
    path = tmp_path / "tok.gguf"
    _write_gguf(path, ["ĠParis", ".", "Ċ", "Hello"])
    tk = nh.Tokenizer.Load(str(path))
    assert tk is not None and tk.vocab_size() == 4
    assert tk.Decode([0, 1]) == " Paris."
    assert tk.Decode([3, 2, 3]) == "Hello\nHello"
    assert tk.Decode([]) == ""
    assert tk.Decode([99]) == ""


def test_encodes_with_bpe_and_round_trips(tmp_path):
    path = tmp_path / "enc.gguf"
    _write_gguf(path, ["h", "i", "hi"], ["h i"])
    tk = nh.Tokenizer.Load(str(path))
    assert tk is not None
    assert tk.Encode("hi") == [2]
    assert tk.Encode("h") == [0]
    assert tk.Decode(tk.Encode("hi")) == "hi"


def test_returns_null_without_vocab(tmp_path):
    path = tmp_path / "novocab.gguf"
    _write_gguf(path, other=1)
    assert nh.Tokenizer.Load(str(path)) is None
    assert nh.Tokenizer.Load(str(tmp_path / "no_such.gguf")) is None
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF\x03\x00\x00\x00")  # truncated header
    assert nh.Tokenizer.Load(str(bad)) is None
    # A string array claiming more entries than the file can hold.
    import struct

    key = b"tokenizer.ggml.tokens"
    huge = tmp_path / "huge.gguf"
    huge.write_bytes(b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + struct.pack("<Q", len(key)) + key +
                     struct.pack("<IIQ", 9, 8, 1 << 27))
    assert nh.Tokenizer.Load(str(huge)) is None


def test_vocabulary_of_another_type_is_no_vocabulary(tmp_path):
    """tokenizer.ggml.tokens must be a string array; merges of another type
    count as absent (tokenizer.cc:74-85)."""
    import gguf

    p1 = tmp_path / "ints.gguf"
    w = gguf.GGUFWriter(str(p1), "olmoe")
    w.add_array("tokenizer.ggml.tokens", [1, 2, 3])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    assert nh.Tokenizer.Load(str(p1)) is None
    p2 = tmp_path / "intmerges.gguf"
    w = gguf.GGUFWriter(str(p2), "olmoe")
    w.add_token_list(["h", "i", "hi"])
    w.add_array("tokenizer.ggml.merges", [7, 8])
    w.add_array("tokenizer.ggml.token_type", [1, 1, 1])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    tk = nh.Tokenizer.Load(str(p2))
    assert tk is not None and tk.vocab_size() == 3 and tk.Encode("hi") == [0, 1]


# ------------------------------------------------------------------ pre-split
def test_split_matches_the_pattern_on_random_text():
    rng = np.random.default_rng(11)
    for _ in range(400):
        text = _text(rng, int(rng.integers(1, 30)))
        assert nh.Tokenizer.Split(text) == split(text), repr(text)


def test_split_edge_cases():
    cases = ["", " ", "\n", "a\nb", "a \nb", "a\n\nb", "a  b", "   ", "'s", "'sam", "'x", "'S", " 's", "x'll'd",
             "1 2  3", " ½", "\t\tz", "z  z", "z\u0085z", " ", "a\r\n\r\nb", "😀😀 😀", "é"]
    for text in cases:
        assert nh.Tokenizer.Split(text) == split(text), repr(text)
    # The reference's search skips what no alternative matches: the newline
    # of "a\nb" belongs to no chunk.
    assert nh.Tokenizer.Split("a\nb") == [(0, 1), (2, 3)]


def test_invalid_utf8_gives_no_ids(trained):
    _, vocab, merges = trained
    tk = nh.Tokenizer.FromLists(vocab, merges)
    for raw in (b"ab\xffcd", b"\xc3", b"\xe2\x82", b"\xed\xa0\x80", b"\xc0\xaf", b"\xf4\x90\x80\x80"):
        assert tk.Encode(raw) == []
        assert nh.Tokenizer.Split(raw) == []


# ------------------------------------------------------------------ encode / decode
def test_encode_matches_oracle_merges(trained):
    _, vocab, merges = trained
    tk = nh.Tokenizer.FromLists(vocab, merges)
    ora = OracleTokenizer(vocab, merges)
    rng = np.random.default_rng(12)
    for _ in range(200):
        text = _text(rng, int(rng.integers(1, 40)))
        ids = tk.Encode(text)
        assert ids == ora.encode(text), repr(text)
        raw = text.encode()
        assert tk.DecodeBytes(ids) == b"".join(raw[a:b] for a, b in split(text))


def test_encode_with_partial_merges_and_missing_tokens(trained):
    """Fewer merges (longer id lists) and a vocabulary without some symbols
    (their pieces yield no id), as the reference's lookups do."""
    _, vocab, merges = trained
    ora_merges = merges[: len(merges) // 3]
    small_vocab = [t if i % 7 else t + "\u0001x" for i, t in enumerate(vocab)]
    rng = np.random.default_rng(13)
    for v, m in ((vocab, ora_merges), (small_vocab, merges)):
        tk = nh.Tokenizer.FromLists(v, m)
        ora = OracleTokenizer(v, m)
        for _ in range(60):
            text = _text(rng, int(rng.integers(1, 25)))
            assert tk.Encode(text) == ora.encode(text), repr(text)


def test_encode_matches_hf_bpe_on_single_spaced_text(trained):
    hf, vocab, merges = trained
    tk = nh.Tokenizer.FromLists(vocab, merges)
    rng = np.random.default_rng(14)
    for _ in range(200):
        text = _text(rng, int(rng.integers(1, 40)), spaces=[" "])
        assert tk.Encode(text) == hf.encode(text).ids, repr(text)


def test_decode_follows_reference_byte_rules():
    """Vocabulary strings of any code points (not only byte-level ones) decode
    as the reference's reader takes them."""
    rng = np.random.default_rng(15)
    alphabet = [chr(c) for c in list(range(0x20, 0x7F)) + list(range(0xA0, 0x180)) + [0x100, 0x120, 0x143, 0x7FF,
                                                                                      0x800, 0x4E2D, 0x1F600]]
    vocab = ["".join(alphabet[rng.integers(len(alphabet))] for _ in range(rng.integers(1, 6))) for _ in range(300)]
    tk = nh.Tokenizer.FromLists(vocab)
    ora = OracleTokenizer(vocab, [])
    for _ in range(100):
        ids = rng.integers(-3, 320, int(rng.integers(0, 12))).tolist()
        assert tk.DecodeBytes(ids) == ora.decode(ids)
    assert tk.token(0) == vocab[0].encode() and tk.token(-1) == b"" and tk.token(300) == b""


def test_c_entries_report_full_counts_and_write_at_most_cap(trained):
    """nh_tokenizer_encode / decode / token / split return the full count and
    write no more than `cap` entries."""
    import ctypes as C

    from nuthatch_b200._lib import lib

    _, vocab, merges = trained
    tk = nh.Tokenizer.FromLists(vocab, merges)
    text = "the quick brown fox jumps over the lazy dog".encode()
    full = tk.Encode(text)
    ids = (C.c_int32 * 8)(*([-7] * 8))
    n = lib().nh_tokenizer_encode(tk._h, text, len(text), ids, 3)
    assert n == len(full) and list(ids[:3]) == full[:3] and list(ids[3:]) == [-7] * 5
    arr = (C.c_int32 * len(full))(*full)
    buf = C.create_string_buffer(b"#" * 16, 16)
    m = lib().nh_tokenizer_decode(tk._h, arr, len(full), buf, 5)
    assert m == len(text) and buf.raw[:5] == text[:5] and buf.raw[5:] == b"#" * 11
    bounds = (C.c_int64 * 4)(*([-1] * 4))
    k = lib().nh_tokenizer_split(text, len(text), bounds, 1)
    assert k == 9 and list(bounds) == [0, 3, -1, -1]
    assert lib().nh_tokenizer_encode(None, text, len(text), None, 0) < 0
    assert lib().nh_tokenizer_from_lists((C.c_char_p * 2)(b"a", None), 2, None, 0) is None
