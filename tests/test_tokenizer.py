"""The byte-level BPE tokenizer (mamba_integer_b200/tokenizer/bpe.cpp, the
reference's Rust tokenizer API) against its oracle (oracle/tokenizer.py: the
same split pattern run by the `regex` module, the same merge and training
loops): pieces, encodings, training, save/load, decoding and the C ABI."""
import os
import random
import re

import pytest

from oracle import tokenizer as ot

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# characters that exercise every branch of the split pattern and every class boundary
POOL = (list("abcXYZ019 '.,!?-_()[]{}\"/\\@#$%^&*+=<>~`|;:") + ["\t", "\r", "\n", "\r\n", "  ", "   "]
        + ["'s", "'S", "'t", "'d", "'m", "'ll", "'LL", "'Ll", "'ve", "'VE", "'re", "'Re", "'ſ", "'x", "'1"]
        + list("éßÆøŁ") + list("αβΓΔ") + list("жЩё") + list("日本語中文") + list("한국어") + list("مرحبا")
        + ["क्ष", "é", "́"]  # Devanagari conjunct, combining acute (a mark: "other")
        + list("١٢٣²³ⅧⅫ༳")  # Nd, No, Nl numbers
        + list("   　\u0085     \u000b\u000c")  # white space
        + list("\u001c\u001f​﻿᠎")  # not white space
        + ["\U0001F600", "\U0001F44D\U0001F3FD", "❤️", "\U00010348", "\U000323B0"])


def _corpus(n, seed=0, maxlen=30):
    rng = random.Random(seed)
    return ["".join(rng.choice(POOL) for _ in range(rng.randint(0, maxlen))) for _ in range(n)]


@pytest.fixture(scope="module")
def tok_cls():
    from mamba_integer_b200 import build
    build.build_bpe()
    from mamba_integer_b200.rust_tokenizer import RustTokenizer
    return RustTokenizer


def test_header_declares_library_exports(tok_cls):
    with open(os.path.join(ROOT, "include", "mi_bpe.h")) as f:
        hdr = f.read()
    declared = set(re.findall(r"\b(tokenizer_\w+|mi_bpe_\w+)\s*\(", hdr))
    t = tok_cls()
    for name in declared:
        assert hasattr(t.lib, name), name
    assert declared == {"tokenizer_new", "tokenizer_free", "tokenizer_train", "tokenizer_encode",
                        "tokenizer_free_ids", "tokenizer_save", "tokenizer_load", "mi_bpe_pretokenize"}


def test_pretokenize_matches_regex_engine(tok_cls):
    t = tok_cls()
    for s in _corpus(3000, seed=1) + ["", " ", "\n", "a", "'", "' ", "'s", "x  ", "  x", " \n ", "1234567"]:
        assert t.pretokenize(s) == ot.pretokenize(s), repr(s)


def test_random_code_points_match_regex_engine(tok_cls):
    # code points drawn from the whole range (surrogates excluded), in runs with spaces and ASCII
    rng = random.Random(7)
    t = tok_cls()
    for _ in range(400):
        cps = []
        for _ in range(rng.randint(1, 24)):
            r = rng.random()
            if r < 0.6:
                cp = rng.randrange(0x110000)
                while 0xD800 <= cp <= 0xDFFF:
                    cp = rng.randrange(0x110000)
            elif r < 0.8:
                cp = rng.choice([0x20, 0x0A, 0x0D, 0x27, 0x73])
            else:
                cp = rng.randrange(0x20, 0x7F)
            cps.append(chr(cp))
        s = "".join(cps).replace("\x00", "")
        assert t.pretokenize(s) == ot.pretokenize(s), repr(s)


def _train_file(tmp_path, lines):
    p = tmp_path / "corpus.txt"
    p.write_text("\n".join(lines) + "\n", encoding="utf-8")
    return str(p)


def test_training_encoding_and_save_load(tok_cls, tmp_path):
    rng = random.Random(3)
    words = ["the", "cat", "sat", "on", "mat", "integer", "mamba", "scan", "don't", "we'll", "2048", "B200",
             "naïve", "日本", "x", "!!", "..."]
    lines = [" ".join(rng.choice(words) for _ in range(rng.randint(1, 12))) for _ in range(300)]
    path = _train_file(tmp_path, lines)
    t = tok_cls()
    t.train(path, 256 + 60)
    merges_ref = ot.train(lines, 256 + 60)
    saved = str(tmp_path / "merges.txt")
    t.save(saved)
    assert ot.load_merges(saved) == merges_ref
    t2 = tok_cls(merges_path=saved)
    for s in lines[:100] + _corpus(200, seed=9):
        ids = t2.encode(s)
        assert ids == ot.encode(s, merges_ref), repr(s)
        assert t2.decode(ids) == s
    with open(saved) as f:
        assert [int(x.split()[1]) for x in f] == sorted(merges_ref.values())


def test_reference_merges_file_if_present(tok_cls):
    path = os.environ.get("MI_REFERENCE_MERGES", "")
    if not path or not os.path.exists(path):
        pytest.skip("set MI_REFERENCE_MERGES to the reference's configs/rust_bpe_merges.txt")
    t = tok_cls(merges_path=path)
    merges = ot.load_merges(path)
    for s in _corpus(500, seed=11, maxlen=60):
        assert t.encode(s) == ot.encode(s, merges), repr(s)


def test_invalid_utf8_and_empty_input(tok_cls):
    import ctypes
    t = tok_cls()
    n = ctypes.c_size_t(5)
    assert not t.lib.tokenizer_encode(t.tokenizer_ptr, b"ab\xffcd", ctypes.byref(n)) and n.value == 0
    assert not t.lib.tokenizer_encode(t.tokenizer_ptr, b"\xed\xa0\x80", ctypes.byref(n))  # a surrogate
    assert not t.lib.tokenizer_encode(t.tokenizer_ptr, b"\xc0\xaf", ctypes.byref(n))  # overlong
    assert t.encode("") == []
    assert t.lib.tokenizer_load(t.tokenizer_ptr, b"/nonexistent/merges.txt") == -1
    assert t.lib.tokenizer_train(t.tokenizer_ptr, b"/nonexistent/corpus.txt", 300) == -1
