"""The .hsm loader of the product (hs_model_check, the checks of hs_model_load on the host) and
the oracle's loader (oracle/hs_model.cpp) on the refusal cases of the reference's own reader
tests, crates/hardshell/tests/hsm.rs:124-321 (bad magic and version, every truncation, trailing
bytes, floats in the header, unknown, missing and duplicate fields, a header that is not UTF-8,
bad model fields, bad tensor entries, a non-canonical layout, non-zero padding, a bad
vocabulary) and security_hsm.rs (long unknown names and values), restated on the conformance
model tiny.hsm (a GPT-2 model with merges, where the reference tests use a bare tensor file).
Every case must be refused by both loaders. Then a seeded sweep of damaged files (byte flips,
cuts, insertions, as crates/hardshell/tests/fuzz_hsm.rs damages files): the two loaders must
agree, refusing or accepting with the same dimensions and hash.

The cases are restated here, not copied: the file edits are those of the reference's `rebuild`
helper (hsm.rs:57-86: a JSON edit, or an edit of the serialised header text, with every section
moved by a multiple of 64 bytes so the layout stays canonical unless the edit changes it).
"""

import json
import struct

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B

from .common import tiny_bytes


def _header_len(f: bytes) -> int:
    return struct.unpack("<I", f[12:16])[0]


def _header(f: bytes) -> dict:
    return json.loads(f[16:16 + _header_len(f)])


def rebuild(orig: bytes, edit_value=None, edit_text=None) -> bytes:
    """orig with its header changed; the sections (vocabulary, merges, tensors) move by the
    smallest multiple of 64 bytes that makes room for the new header text."""
    base = _header(orig)
    voff = base["vocabulary"]["offset"]
    for k in range(256):
        v = json.loads(json.dumps(base))
        shift = 64 * k
        v["vocabulary"]["offset"] += shift
        if "merges" in v:
            v["merges"]["offset"] += shift
        for t in v["tensors"]:
            t["offset"] += shift
        if edit_value:
            edit_value(v)
        text = json.dumps(v, separators=(",", ":"), ensure_ascii=False)
        if edit_text:
            text = edit_text(text)
        raw = text.encode()
        room = voff + shift - 16
        if len(raw) <= room:
            return orig[:12] + struct.pack("<I", room) + raw + b" " * (room - len(raw)) + orig[voff:]
    raise AssertionError("the header does not fit")


def product_refuses(f: bytes) -> bool:
    try:
        B.check_model(f)
    except B.HardShellError as e:
        assert e.code == B.HS_MODEL, e
        return True
    return False


def oracle_refuses(f: bytes) -> bool:
    try:
        O.Model(f)
    except O.OracleError:
        return True
    return False


def refused(f: bytes):
    assert product_refuses(f), "the product loader accepted the file"
    assert oracle_refuses(f), "the oracle loader accepted the file"


def _set(path, value):
    def edit(v):
        d = v
        for k in path[:-1]:
            d = d[k]
        d[path[-1]] = value
    return edit


def _drop(path):
    def edit(v):
        d = v
        for k in path[:-1]:
            d = d[k]
        del d[path[-1]]
    return edit


@pytest.fixture(scope="module")
def tiny():
    return tiny_bytes()


def test_both_loaders_accept_the_file_and_a_rebuild_without_edits(tiny):
    info = B.check_model(tiny)
    assert (info["n_layer"], info["d_model"], info["vocab"], info["n_ctx"]) == (2, 64, 300, 64)
    same = rebuild(tiny)
    assert B.check_model(same)["vocab"] == 300
    O.Model(same)


def test_bad_magic_and_version(tiny):
    refused(b"X" + tiny[1:])
    for version in (0, 3):
        refused(tiny[:8] + struct.pack("<I", version) + tiny[12:])
    # Version 2 exists, but this file has no part that needs it (hsm.rs:131-133).
    refused(tiny[:8] + struct.pack("<I", 2) + tiny[12:])


def test_every_truncation_and_trailing_bytes(tiny):
    hl = _header_len(tiny)
    cuts = list(range(0, 16 + hl + 64)) + list(range(16 + hl + 64, len(tiny), 997)) + [len(tiny) - 1]
    for n in cuts:
        assert product_refuses(tiny[:n]), n
        assert oracle_refuses(tiny[:n]), n
    refused(tiny + b"\0")


def test_floats_in_the_header(tiny):
    refused(rebuild(tiny, _set(["model", "n_layer"], 2.0)))
    refused(rebuild(tiny, edit_text=lambda t: t.replace('"eot_token":299', '"eot_token":299e0')))
    refused(rebuild(tiny, edit_text=lambda t: t.replace('"ln_k":48', '"ln_k":4.8e1')))
    refused(rebuild(tiny, edit_value=lambda v: v["tensors"][0].__setitem__("shape", [300.0, 64])))
    refused(rebuild(tiny, _set(["model", "n_head"], -4)))
    refused(rebuild(tiny, _set(["model", "n_head"], 18_446_744_073_709_551_616)))


def test_unknown_missing_and_duplicate_fields(tiny):
    refused(rebuild(tiny, _set(["model", "dropout"], 0)))
    refused(rebuild(tiny, _set(["extra"], 1)))
    refused(rebuild(tiny, _drop(["model", "d_ff"])))
    refused(rebuild(tiny, edit_text=lambda t: t.replace('"n_layer":2', '"n_layer":2,"n_layer":2')))
    refused(rebuild(tiny, edit_value=lambda v: v["tensors"][1].__setitem__("scale", 1)))
    # security_hsm.rs: a long unknown field name and a long string value are refused (and the
    # reference keeps its message short; the refusal is what both loaders share).
    refused(rebuild(tiny, _set(["model", "x" * 5000], 0)))
    refused(rebuild(tiny, _set(["model", "architecture"], "g" * 5000)))


def test_a_header_that_is_not_utf8(tiny):
    good = rebuild(tiny, edit_text=lambda t: t.replace('"gpt2"', '"gpté"'))
    refused(good)  # valid UTF-8, refused for its architecture name
    bad = bytearray(good)
    pos = bytes(bad).index(b"\xc3\xa9")
    bad[pos] = 0xFF
    refused(bytes(bad))


def test_bad_model_fields(tiny):
    refused(rebuild(tiny, _set(["model", "eot_token"], 300)))
    refused(rebuild(tiny, _set(["model", "vocab_size"], 0)))
    refused(rebuild(tiny, _set(["model", "constants", "ln_k"], 49)))
    refused(rebuild(tiny, _set(["model", "constants", "ln_eps"], 0)))
    refused(rebuild(tiny, _set(["model", "constants", "softmax_p"], 31)))
    refused(rebuild(tiny, _set(["model", "architecture"], "GPT2")))
    refused(rebuild(tiny, edit_value=lambda v: v["tensors"][0].__setitem__("name", "")))
    refused(rebuild(tiny, _set(["model", "n_head"], 3)))  # d_model 64 is not a multiple of 3
    refused(rebuild(tiny, _set(["model", "n_layer"], 3)))  # the tensors of layer 2 are missing


def test_bad_tensor_entries(tiny):
    t0 = lambda k, x: (lambda v: v["tensors"][0].__setitem__(k, x))  # noqa: E731
    t1 = lambda k, x: (lambda v: v["tensors"][1].__setitem__(k, x))  # noqa: E731
    refused(rebuild(tiny, t0("dtype", "f32")))
    refused(rebuild(tiny, t0("dtype", "i16")))
    refused(rebuild(tiny, t0("shape", [150, 128])))
    refused(rebuild(tiny, t0("shape", [300, 0])))
    refused(rebuild(tiny, t0("shape", [])))
    refused(rebuild(tiny, t0("shift", 3)))  # wte has no rescale shift
    refused(rebuild(tiny, t1("length", 4)))
    refused(rebuild(tiny, t1("name", "w")))  # an unexpected tensor
    refused(rebuild(tiny, _drop(["tensors", 1])))  # a missing tensor
    refused(rebuild(tiny, t1("shift", 256)))  # a shift is a u8 (header.rs:182)
    refused(rebuild(tiny, t1("shift", -1)))


def test_a_non_canonical_layout(tiny):
    def move(path, delta):
        def edit(v):
            d = v
            for k in path[:-1]:
                d = d[k]
            d[path[-1]] += delta
        return edit

    refused(rebuild(tiny, move(["tensors", 1, "offset"], 64)))
    refused(rebuild(tiny, move(["tensors", 1, "offset"], -64)))
    refused(rebuild(tiny, move(["vocabulary", "offset"], 64)))
    refused(rebuild(tiny, move(["merges", "offset"], 64)))
    refused(rebuild(tiny, move(["tensors", 3, "offset"], 1)))


def test_non_zero_padding(tiny):
    v = _header(tiny)
    t0 = v["tensors"][0]
    gap = t0["offset"] + t0["length"]
    nxt = v["tensors"][1]["offset"]
    if gap < nxt:  # the padding after wte
        bad = bytearray(tiny)
        bad[gap] = 1
        refused(bytes(bad))
    vend = v["vocabulary"]["offset"] + v["vocabulary"]["length"]
    if vend < v["merges"]["offset"]:  # the padding between the vocabulary and the merges
        bad = bytearray(tiny)
        bad[vend] = 1
        refused(bytes(bad))


def test_a_bad_vocabulary(tiny):
    refused(rebuild(tiny, _set(["model", "vocab_size"], 299)))  # one token fewer than the file
    voff = _header(tiny)["vocabulary"]["offset"]
    bad = bytearray(tiny)
    bad[voff] = 200  # a token length that runs past the section
    bad[voff + 1] = 200
    refused(bytes(bad))


def test_bad_merges(tiny):
    v = _header(tiny)
    moff = v["merges"]["offset"]
    first = struct.unpack("<II", tiny[moff:moff + 8])
    # An id out of the vocabulary, a pair whose joined bytes are no token, a duplicate pair.
    for pair in [(300, first[1]), (first[1], first[0] if first[0] != first[1] else 0)]:
        bad = bytearray(tiny)
        bad[moff:moff + 8] = struct.pack("<II", *pair)
        if bytes(bad) != tiny:
            refused(bytes(bad))
    second = struct.unpack("<II", tiny[moff + 8:moff + 16])
    if second != first:
        bad = bytearray(tiny)
        bad[moff + 8:moff + 16] = struct.pack("<II", *first)
        refused(bytes(bad))
    refused(rebuild(tiny, _set(["merges", "length"], v["merges"]["length"] - 4)))


def test_damaged_files_are_refused_or_read_alike():
    """Seeded damage (fuzz_hsm.rs): byte flips, cuts and insertions anywhere in the file. Both
    loaders refuse, or both accept with the same dimensions and hash."""
    tiny = tiny_bytes()
    rng = np.random.default_rng(0x45A)
    accepted = 0
    for case in range(300):
        f = bytearray(tiny)
        kind = case % 3
        pos = int(rng.integers(0, len(f)))
        if kind == 0:
            f[pos] ^= int(rng.integers(1, 256))
        elif kind == 1:
            del f[pos:pos + int(rng.integers(1, 9))]
        else:
            f[pos:pos] = bytes(rng.integers(0, 256, int(rng.integers(1, 9)), dtype=np.uint8))
        f = bytes(f)
        p, o = product_refuses(f), oracle_refuses(f)
        assert p == o, (case, kind, pos)
        if not p:
            accepted += 1
            info = B.check_model(f)
            om = O.Model(f)
            assert (info["vocab"], info["n_ctx"], info["d_model"]) == (om.vocab, 64, 64)
    assert accepted < 300
