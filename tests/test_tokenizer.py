"""The fold's tokenizer (hs_tokenizer_*: crates/taco/src/tokenizer), host code, on the CPU.

Pinned two ways: the pre-tokenizer on the piece vectors of the reference's own tests
(crates/taco/src/tokenizer/pretokenize.rs tests), and the whole tokenizer on the token streams
inside the published coded blocks of the conformance containers, which the reference's tokenizer
made (each coded block is decoded with the oracle and its tokens compared with the tokens of its
original bytes). Round trips cover ill-formed UTF-8 and every byte value.
"""

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import container as C

from .common import GOLDEN, tiny_bytes

# crates/taco/src/tokenizer/pretokenize.rs, tests.
PIECES = [
    ("Hello world", ["Hello", " world"]),
    ("  two  spaces", [" ", " two", " ", " spaces"]),
    ("don't we'll", ["don", "'t", " we", "'ll"]),
    ("\"'s", ["\"'", "s"]),
    ("'S", ["'", "S"]),
    ("a\n\n b", ["a", "\n\n", " b"]),
    ("a\tb", ["a", "\t", "b"]),
    ("a   ", ["a", "   "]),
    (" ", [" "]),
    ("x \n", ["x", " \n"]),
    ("abc123!?", ["abc", "123", "!?"]),
    (" 42 ++", [" 42", " ++"]),
    ("हि", ["ह", "ि"]),  # a Devanagari vowel sign is not a letter
]


@pytest.fixture(scope="module")
def tok():
    t = B.Tokenizer(tiny_bytes())
    yield t
    t.close()


@pytest.mark.parametrize("text,want", PIECES)
def test_pieces_follow_the_gpt2_pattern(tok, text, want):
    assert [p.decode() for p in tok.pieces(text.encode())] == want


def test_pieces_never_cross_an_ill_formed_byte(tok):
    # 0xFF and a truncated 3-byte sequence split the runs; each of their bytes is a piece.
    data = b"ab\xffcd \xe2\x82 ef\xe2\x82\xac"
    assert tok.pieces(data) == [b"ab", b"\xff", b"cd", b" ", b"\xe2", b"\x82", b" ef", b"\xe2\x82\xac"]


@pytest.mark.parametrize("name", ["predicted_text_k0", "predicted_text_k32", "all_kinds_text"])
def test_tokens_of_the_published_coded_blocks(tok, name):
    om = O.Model(tiny_bytes())
    c = C.parse((GOLDEN / (name + ".taco")).read_bytes())
    data = (GOLDEN / (name + ".in")).read_bytes()
    off, checked = 0, 0
    for b in c.blocks:
        orig = data[off:off + b.original_len]
        off += b.original_len
        if b.kind != C.KIND_CODED:
            continue
        got_bytes, tokens = O.decode_block(om, b.stored, b.original_len, c.overlap)
        assert got_bytes == orig
        assert tok.encode(orig).tolist() == list(tokens)
        checked += 1
    assert checked > 0


def test_any_bytes_round_trip(tok):
    om = O.Model(tiny_bytes())
    rng = np.random.default_rng(3)
    cases = [b"", bytes(range(256)), "héllo wörld — ünïcödé ✓ 😀".encode(), b"\xed\xa0\x80\xf4\x90\x80\x80"]
    cases += [rng.integers(0, 256, n, dtype=np.uint8).tobytes() for n in (1, 7, 100, 3000)]
    cases += [bytes(rng.choice(list(b"ab c'\n\t1"), 500)) for _ in range(3)]
    for data in cases:
        toks = tok.encode(data)
        assert b"".join(om.token_bytes(int(t)) for t in toks) == data
        assert toks.size <= len(data)


def test_a_bad_model_file_is_refused():
    with pytest.raises(B.HardShellError) as e:
        B.Tokenizer(b"not a model")
    assert e.value.code == B.HS_MODEL
