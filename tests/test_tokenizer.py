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


# ---- the Unicode classes: the reference's own tables ----

# The counts of the three tables of the reference's crates/taco/src/tokenizer/unicode_tables.rs
# (LETTER :12-15, NUMBER :168-171, WHITESPACE :207-210), and the SHA-256 of their ranges written
# as "LO-HI;" in hex, in order (the digest gen_unicode_classes.py records).
REFERENCE_TABLES = {
    "kLetter": (694, 158172, "7e16409502d0aeccb1c6e18a1f43d85b4afca5c041901f5c0b9d3ff31cb8ad43"),
    "kNumber": (148, 2247, "63534d2a58d9ce4ddafb45b3819baa5c05459365d2a5d070277ea389d4d15c1c"),
    "kWhiteSpace": (10, 25, "263aa7d5325ac8ea2f2b9627c44ce959bc2af786386e205068c76ccbe65f16f3"),
}


def _inc_tables() -> dict[str, list[tuple[int, int]]]:
    import re
    from pathlib import Path

    text = (Path(B.__file__).resolve().parent / "csrc" / "hs_unicode.inc").read_text()
    out = {}
    for m in re.finditer(r"static const CodeRange (\w+)\[\] = \{(.*?)\};", text, re.S):
        out[m.group(1)] = [(int(a, 16), int(b, 16)) for a, b in re.findall(r"\{0x([0-9A-F]+), 0x([0-9A-F]+)\}",
                                                                           m.group(2))]
    return out


def test_unicode_tables_are_the_reference_tables():
    import hashlib

    tables = _inc_tables()
    for name, (n_ranges, n_points, sha) in REFERENCE_TABLES.items():
        rs = tables[name]
        assert len(rs) == n_ranges, name
        assert sum(b - a + 1 for a, b in rs) == n_points, name
        assert hashlib.sha256("".join(f"{a:X}-{b:X};" for a, b in rs).encode()).hexdigest() == sha, name


def test_pieces_follow_the_reference_classes_where_this_image_differs(tok):
    """Every code point that the reference's tables and this image's `regex` module classify
    differently: the pieces around it follow the reference's class (a letter joins letters, a
    number joins numbers, any other non-space joins punctuation, and none of them joins another
    class), as pretokenize.rs does with those tables."""
    regex = pytest.importorskip("regex")
    tables = _inc_tables()

    def member(rs, c):
        import bisect
        i = bisect.bisect_right(rs, (c, 0x110000)) - 1
        return i >= 0 and rs[i][0] <= c <= rs[i][1]

    rx_l, rx_n = regex.compile(r"\p{L}"), regex.compile(r"\p{N}")
    rep = {"L": "a", "N": "1", "O": "!"}
    differ = 0
    for c in range(0x80, 0x110000):
        if 0xD800 <= c <= 0xDFFF or member(tables["kWhiteSpace"], c):
            continue
        ref = "L" if member(tables["kLetter"], c) else "N" if member(tables["kNumber"], c) else "O"
        ch = chr(c)
        img = "L" if rx_l.match(ch) else "N" if rx_n.match(ch) else "O"
        if ref == img:
            continue
        differ += 1
        same = (rep[ref] + ch + rep[ref]).encode()
        assert tok.pieces(same) == [same], hex(c)
        for other in "LNO":
            if other != ref:
                text = (rep[other] + ch).encode()
                assert tok.pieces(text) == [rep[other].encode(), ch.encode()], (hex(c), other)
    # This image's regex 2026.3.32 knows an older Unicode than the reference's tables: 12,500
    # letters and 323 numbers are new there. A newer regex would leave fewer to check.
    print(f"{differ} code points classified by the reference's tables, not this image's regex")


# ---- the refusals of the fold on several GPUs, decided on the host before any GPU call ----

def test_fold_multi_refuses_a_bad_model_file(tok):
    with pytest.raises(B.HardShellError) as e:
        B.fold_multi([0], b"not a model", tok, b"some text", 300, 0, slots=2, max_rows=64)
    assert e.value.code == B.HS_MODEL


def test_fold_multi_refuses_a_tokenizer_of_another_vocabulary(tok):
    from taco_b200 import synth

    other = synth.gpt2_hsm(7, shape=synth.MINI)  # 1,000 tokens; the tiny model has 300
    with pytest.raises(B.HardShellError) as e:
        B.fold_multi([0], other, tok, b"some text", 300, 0, slots=2, max_rows=64)
    assert e.value.code == B.HS_MODEL
    assert "TokenizerMismatch" in str(e.value)


def test_fold_multi_with_no_gpu_that_opens_fails_with_the_open_error(tok, monkeypatch):
    monkeypatch.setenv("HS_FAIL_OPEN", "0,1")
    with pytest.raises(B.HardShellError) as e:
        B.fold_multi([0, 1], tiny_bytes(), tok, b"some text " * 100, 300, 0, slots=2, max_rows=64)
    assert e.value.code == B.HS_NO_DEVICE
    assert "no GPU of the fold opened" in str(e.value)


# ---- the synthetic GPT-2 vocabulary of the benchmark: byte-level BPE with merges ----

def test_synthetic_vocabulary_tokenizes_the_zipf_text_as_the_python_bpe():
    """The product tokenizer, on the merges section of the synthetic GPT-2 model, gives the tokens
    of the Python restatement of the BPE (taco_b200/synth.py tokenize_text) for Zipf text, and
    every " w" word of the text is one token."""
    from taco_b200 import synth

    model = synth.gpt2_hsm(124)
    t = B.Tokenizer(model)
    try:
        vocab = synth.vocabulary()
        merge_list = synth.merges(vocab)
        assert len(merge_list) == len(vocab) - 257
        text = synth.zipf_text(300_000, seed=11)
        got = t.encode(text)
        want = synth.tokenize_text(text, vocab, merge_list)
        assert np.array_equal(got, want)
        words = set(synth.text_word_ids(vocab).tolist())
        n_space_words = text.count(b" ")
        assert sum(1 for x in got.tolist() if x in words) == n_space_words
        assert b"".join(vocab[x] for x in got.tolist()) == text
    finally:
        t.close()


def test_unfold_multi_refusals_before_any_gpu(tok, monkeypatch):
    good = (GOLDEN / "predicted_text_k32.taco").read_bytes()
    with pytest.raises(B.HardShellError) as e:
        B.unfold_multi([0], b"not a model", tok, good)
    assert e.value.code == B.HS_MODEL
    monkeypatch.setenv("HS_FAIL_OPEN", "0")
    with pytest.raises(B.HardShellError) as e:
        B.unfold_multi([0], tiny_bytes(), tok, good)
    assert e.value.code == B.HS_NO_DEVICE
