"""The container rules of the unfold, one at a time, on the host (no GPU): each case breaks one rule
of crates/taco-format (header.rs:220-330, reader.rs) in a valid container. The library's reader
refuses it with HS_FORMAT before any output, and container.py's parser, the repository's other
restatement of the same rules, refuses it too. The valid container unfolds.
"""

import hashlib

import pytest

from taco_b200 import backend as B
from taco_b200 import container as C

from .common import tiny_bytes

MODEL_HASH = hashlib.sha256(tiny_bytes()).digest()


def _header_set(blob: bytes, at: int, value: bytes) -> bytes:
    b = bytearray(blob)
    b[at:at + len(value)] = value
    return bytes(b)


def _cases():
    """(name, container bytes, substring of the library's message)."""
    text = b"a" * 200
    frame = _zstd_rle(text[100:])
    c = C.Container(2, MODEL_HASH, 200, hashlib.sha256(text).digest(), 100)
    c.blocks = [C.Block(0, C.KIND_RAW, 100, text[:100]), C.Block(1, C.KIND_ZSTD, 100, frame)]
    good = C.build(c)
    H = C.HEADER_LEN
    cases = [
        ("bad magic", b"TACX" + good[4:], "bad magic"),
        ("version 3", _header_set(good, 4, (3).to_bytes(2, "little")), "unsupported version"),
        ("flags", _header_set(good, 6, (1).to_bytes(2, "little")), "unknown flags"),
        ("block size 0", _header_set(good, 80, (0).to_bytes(4, "little")), "block size"),
        ("block size past 64 MiB", _header_set(good, 80, ((64 << 20) + 1).to_bytes(4, "little")), "block size"),
        ("block count", _header_set(good, 84, (3).to_bytes(4, "little")), "block count"),
        ("profile 2", _header_set(good, 88, b"\x02"), "version 2 fields"),
        ("reserved byte", _header_set(good, 89, b"\x01"), "version 2 fields"),
        ("unknown coding part", _header_set(good, 90, (4).to_bytes(2, "little")), "version 2 fields"),
        ("text profile with the mixer bit", _header_set(good, 90, (1).to_bytes(2, "little")), "no mixer"),
        ("mixer rule without the mixer bit", _header_set(good, 92, b"\x01"), "mixer rule"),
        ("overlap bit with K = 0", _header_set(good, 90, (2).to_bytes(2, "little")), "overlap"),
        ("K without the overlap bit", _header_set(good, 94, (5).to_bytes(2, "little")), "overlap"),
        ("coding parameter byte 1", _header_set(good, 93, b"\x01"), "coding parameters"),
        ("coding parameter byte 11", _header_set(good, 103, b"\x01"), "coding parameters"),
        ("block kind 4", _header_set(good, H + 5, b"\x04"), "kind"),
        ("raw block of another length", _header_set(good, H + 1, (99).to_bytes(4, "little")), "raw block"),
        ("zstd block not smaller", _header_set(good, H + 6, (100).to_bytes(4, "little")), "not smaller"),
        ("truncated table", good[:H + 7], "truncated"),
    ]
    # A coded block in a container that names no model.
    nm = C.Container(2, bytes(32), 200, hashlib.sha256(text).digest(), 100)
    nm.blocks = [C.Block(0, C.KIND_RAW, 100, text[:100]), C.Block(1, C.KIND_CODED, 100, b"\x05abc")]
    cases.append(("coded block without a model", C.build(nm), "needs a model"))
    # A mixed block without the mixer bit (profile logs, no mixer rule).
    mx = C.Container(2, MODEL_HASH, 200, hashlib.sha256(text).digest(), 100, profile=C.PROFILE_LOGS)
    mx.blocks = [C.Block(0, C.KIND_RAW, 100, text[:100]), C.Block(1, C.KIND_MIXED, 100, b"\x05abc")]
    cases.append(("mixed block without the mixer bit", C.build(mx), "mixer bit"))
    return good, text, cases


def _zstd_rle(data: bytes) -> bytes:
    """One zstd frame of a run of one byte value repeated (RFC 8878: a 1-byte content size and an
    RLE block); `data` must be one byte value repeated."""
    assert len(set(data)) == 1 and len(data) < 256
    header = bytes([0x28, 0xB5, 0x2F, 0xFD, 0x20, len(data)])  # magic, single segment, content size
    block = (1 | (1 << 1) | (len(data) << 3)).to_bytes(3, "little")  # the last block, RLE, its length
    return header + block + data[:1]


@pytest.fixture(scope="module")
def tok():
    t = B.Tokenizer(tiny_bytes())
    yield t
    t.close()


def test_the_valid_container_unfolds(tok, monkeypatch):
    monkeypatch.setenv("HS_FAIL_OPEN", "0")
    good, text, _ = _cases()
    assert C.parse(good).blocks[1].kind == C.KIND_ZSTD
    assert B.unfold_multi([0], tiny_bytes(), tok, good) == text


@pytest.mark.parametrize("name", [c[0] for c in _cases()[2]])
def test_each_broken_rule_is_a_format_error(tok, monkeypatch, name):
    monkeypatch.setenv("HS_FAIL_OPEN", "0")
    _, _, cases = _cases()
    blob, why = next((b, w) for n, b, w in cases if n == name)
    with pytest.raises(C.FormatError):
        C.parse(blob)
    out = []
    with pytest.raises(B.HardShellError) as e:
        B.unfold_pipe_multi([0], tiny_bytes(), tok, _reader(blob), out.append)
    assert e.value.code == B.HS_FORMAT and why in str(e.value), str(e.value)
    assert out == []


def _reader(data: bytes):
    pos = [0]

    def read(n):
        piece = data[pos[0]:pos[0] + n]
        pos[0] += len(piece)
        return piece

    return read
