"""Tokenizer (g2_tokenizer_*, the CLI text path) against the reference's own
tokenizer.c (tokenizer.c:442-579).

* golden: tests/golden/tok/ holds a synthetic byte-level BPE vocabulary in
  GPT-2's formats and, per case text, the ids and decoded bytes produced by
  the reference's tokenizer (tests/golden/make_tokenizer_fixture.py) -- ours
  must give the same ids (also when truncated to 8) and bytes;
* fuzz: random byte strings compared with the reference library directly,
  when oracle/_ref is built;
* properties: decode(encode(text)) == text (every byte has a symbol), ids in
  range, argument and file errors.
"""
import json
import os
import random

import pytest

import oracle
from gpt2b200 import G2Error, Tokenizer

HERE = os.path.dirname(os.path.abspath(__file__))
TOK = os.path.join(HERE, "golden", "tok")
CASES = json.load(open(os.path.join(TOK, "cases.json")))["cases"]


@pytest.fixture(scope="module")
def tok():
    t = Tokenizer(TOK)
    yield t
    t.close()


@pytest.mark.parametrize("i", range(len(CASES)))
def test_matches_reference_golden(tok, i):
    c = CASES[i]
    data = bytes.fromhex(c["text_hex"])
    ids = tok.encode(data)
    assert ids == c["ids"]
    assert tok.encode(data, 8) == c["ids_max8"]
    assert tok.decode(ids) == bytes.fromhex(c["decoded_hex"])


def test_round_trip_and_range(tok):
    V = tok.vocab_size
    for c in CASES:
        data = bytes.fromhex(c["text_hex"])
        ids = tok.encode(data)
        assert all(0 <= t < V for t in ids)
        assert tok.decode(ids) == data


def _random_text(rng):
    pieces = ["'s", "'re", "'ll", "'t", " ", "  ", "\t", "\n", "x", "ka", "To", "123", "4", "!", "?!", ".", "é", "日",
              "\U0001F642", "'", "ne", "qu", " 9", " a", "--"]
    s = "".join(rng.choice(pieces) for _ in range(rng.randint(0, 40)))
    if rng.random() < 0.3:   # raw bytes, including invalid UTF-8
        s = s.encode() + bytes(rng.randrange(1, 256) for _ in range(rng.randint(1, 8)))
        return s
    return s.encode()


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (reference sources absent)")
def test_fuzz_against_reference_library(tok):
    ref = oracle.RefTokenizer(TOK)
    rng = random.Random(7)
    try:
        for _ in range(400):
            data = _random_text(rng)
            ids = ref.encode(data)
            assert tok.encode(data) == ids, data
            assert tok.decode(ids) == ref.decode(ids)
            n = rng.randint(1, 6)
            assert tok.encode(data, n) == ref.encode(data, n)
        # decoding arbitrary ids, unknown ones included, and a tight output buffer
        for _ in range(100):
            ids = [rng.randrange(-3, tok.vocab_size + 5) for _ in range(rng.randint(0, 30))]
            assert tok.decode(ids) == ref.decode(ids)
            assert tok.decode(ids, 7) == ref.decode(ids, 7)
    finally:
        ref.close()


def test_errors(tmp_path):
    with pytest.raises(G2Error):
        Tokenizer(str(tmp_path))   # no files
    (tmp_path / "vocab.json").write_text('{"a": 0, "b": ')
    (tmp_path / "merges.txt").write_text("#version: 0.2\na b\n")
    t = Tokenizer(str(tmp_path))   # a value-less last entry parses as id 0, as in the reference
    t.close()
    (tmp_path / "vocab.json").write_text('{"a": 0, "b" 1}')
    with pytest.raises(G2Error):
        Tokenizer(str(tmp_path))
