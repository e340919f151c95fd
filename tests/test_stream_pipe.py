"""The stream forms of the fold and unfold (crates/taco/src/stream.rs: StreamFold::to_seekable
and to_writer, the method "spool"; StreamUnfold::from_seekable and from_reader) and the container
checks of the unfold, on the host, with no GPU.

The multi-GPU entry points open their GPUs only when a model window or a coded block needs one,
so two kinds of input run here with every GPU refused (HS_FAIL_OPEN, a host-side refusal):
- a fold in blocks of one byte: a block whose token count already takes its whole length never
  starts a model window (the stop rule, crates/taco/src/codec.rs:70-131), so every block is raw;
- the unfold of the conformance containers whose blocks are raw or zstd.
The spooled container must be the container that container.py builds from the same blocks, with
the input length known or not, across several segments (4,096 blocks each), and its spool files
must never be visible in the spool directory; the seekable outputs must give the same bytes. The
pipe unfold must give the published inputs, and report a missing byte where it is found and an
extra byte at the end, as the reference does. The damaged headers, the version 1 container and
the zstd frame cases follow the reference's stream and security tests
(crates/taco-cli/tests/stream.rs, crates/taco/tests/security_unfold.rs). The one-batch wrappers,
which otherwise run only on a GPU, are checked to reach the library.
"""

import ctypes
import hashlib
import os

import numpy as np
import pytest

from taco_b200 import backend as B
from taco_b200 import container as C

from .common import GOLDEN, tiny_bytes

NO_CODED = ["empty", "one_byte", "random_raw", "text_k0", "text_k20", "text_kinds"]


@pytest.fixture(scope="module")
def tok():
    t = B.Tokenizer(tiny_bytes())
    yield t
    t.close()


@pytest.fixture(autouse=True)
def no_gpu(monkeypatch):
    monkeypatch.setenv("HS_FAIL_OPEN", "0,1")


def _reader(data: bytes, seed: int = 5):
    """read(n) over `data` in pieces of random sizes (a pipe gives what it has)."""
    rng = np.random.default_rng(seed)
    pos = [0]

    def read(n):
        k = min(n, int(rng.integers(1, 5000)))
        out = data[pos[0]:pos[0] + k]
        pos[0] += len(out)
        return out

    return read


def _raw_container(data: bytes) -> bytes:
    """The container of `data` in raw blocks of one byte (the tiny model named, no overlap)."""
    c = C.Container(2, hashlib.sha256(tiny_bytes()).digest(), len(data), hashlib.sha256(data).digest(), 1)
    c.blocks = [C.Block(i, C.KIND_RAW, 1, data[i:i + 1]) for i in range(len(data))]
    return C.build(c)


def _spool(tok, data, length, spool_dir, **kw):
    out = bytearray()
    n, stats = B.fold_spool_multi([0, 1], tiny_bytes(), tok, _reader(data), out.extend, length=length,
                                  spool_dir=spool_dir, block_size=1, **kw)
    assert n == len(out)
    return bytes(out), stats


@pytest.mark.parametrize("size", [0, 1, 4096, 8192, 10_000])
@pytest.mark.parametrize("known", [True, False])
def test_spool_fold_gives_the_container_of_its_blocks(tok, tmp_path, size, known):
    data = np.random.default_rng(size).integers(0, 256, size, dtype=np.uint8).tobytes()
    got, stats = _spool(tok, data, len(data) if known else None, tmp_path)
    assert got == _raw_container(data)
    assert stats["original_len"] == size and stats["blocks"] == size and stats["block_size"] == 1
    assert stats["coded_blocks"] == 0 and stats["gpu_rows"] == 0 and stats["gpus_failed"] == 2
    assert list(tmp_path.iterdir()) == []
    c = C.parse(got)
    assert b"".join(b.stored for b in c.blocks) == data


def test_spool_files_never_show_in_the_directory(tok, tmp_path):
    """The spool files are unlinked as soon as they are made: the directory is empty while the
    container goes out, and after."""
    data = bytes(range(256)) * 40
    seen = []

    def write(chunk):
        seen.append(sorted(p.name for p in tmp_path.iterdir()))

    B.fold_spool_multi([0], tiny_bytes(), tok, _reader(data), write, spool_dir=tmp_path, block_size=1)
    assert seen and all(s == [] for s in seen)


def test_spool_fold_with_the_default_directory(tok, tmp_path, monkeypatch):
    monkeypatch.setenv("TMPDIR", str(tmp_path))
    data = b"pipe" * 3000
    got, _ = _spool(tok, data, None, None)
    assert got == _raw_container(data)


def test_spool_fold_refusals(tok, tmp_path):
    data = b"x" * 5000
    # A known length that the source does not have: fewer or more bytes.
    for length in (len(data) + 1, len(data) - 1):
        with pytest.raises(B.HardShellError) as e:
            _spool(tok, data, length, tmp_path)
        assert e.value.code == B.HS_IO
    # A source or a writer that fails.
    def bad_read(n):
        raise OSError("gone")

    with pytest.raises(B.HardShellError) as e:
        B.fold_spool_multi([0], tiny_bytes(), tok, bad_read, lambda c: None, spool_dir=tmp_path, block_size=1)
    assert e.value.code == B.HS_IO

    def bad_write(chunk):
        raise OSError("disk full")

    with pytest.raises(B.HardShellError) as e:
        B.fold_spool_multi([0], tiny_bytes(), tok, _reader(data), bad_write, spool_dir=tmp_path, block_size=1)
    assert e.value.code == B.HS_IO and "output writer" in str(e.value)
    # A spool directory that does not exist.
    with pytest.raises(B.HardShellError) as e:
        B.fold_spool_multi([0], tiny_bytes(), tok, _reader(data), lambda c: None,
                           spool_dir=tmp_path / "missing", block_size=1)
    assert e.value.code == B.HS_IO and "temporary file" in str(e.value)
    assert list(tmp_path.iterdir()) == []
    # A seekable output needs the length before the first block.
    with pytest.raises(B.HardShellError) as e:
        B.fold_stream_multi([0], tiny_bytes(), tok, B.LEN_UNKNOWN, _reader(data), lambda at, c: None, 1, 0)
    assert e.value.code == B.HS_BAD_ARGUMENT


def test_spool_fold_that_needs_a_window_fails_with_no_gpu(tok, tmp_path):
    """Blocks of 300 bytes of text need the model: with every GPU refused the fold fails with the
    open error, and leaves no spool file."""
    data = (GOLDEN / "text_kinds.in").read_bytes()
    with pytest.raises(B.HardShellError) as e:
        B.fold_spool_multi([0, 1], tiny_bytes(), tok, _reader(data), lambda c: None, spool_dir=tmp_path,
                           block_size=300)
    assert e.value.code == B.HS_NO_DEVICE and "no GPU of the fold opened" in str(e.value)
    assert list(tmp_path.iterdir()) == []


def _unpipe(tok, container: bytes, seed: int = 3):
    out = bytearray()
    n = B.unfold_pipe_multi([0, 1], tiny_bytes(), tok, _reader(container, seed), out.extend)
    return n, bytes(out)


@pytest.mark.parametrize("name", NO_CODED)
def test_pipe_unfold_gives_the_published_input(tok, name):
    container = (GOLDEN / (name + ".taco")).read_bytes()
    want = (GOLDEN / (name + ".in")).read_bytes()
    for seed in (1, 2):
        n, got = _unpipe(tok, container, seed)
        assert n == len(want) and got == want


@pytest.mark.parametrize("known", [True, False])
def test_spool_then_pipe_round_trips_across_segments(tok, tmp_path, known):
    data = np.random.default_rng(9).integers(0, 256, 9_999, dtype=np.uint8).tobytes()
    folded, _ = _spool(tok, data, len(data) if known else None, tmp_path)
    n, got = _unpipe(tok, folded)
    assert n == len(data) and got == data


def test_pipe_unfold_finds_a_missing_byte_where_it_is_needed(tok, tmp_path):
    """A container cut inside its third segment: the first two segments (8,192 bytes) are
    restored before the error, as from_reader restores them."""
    data = np.random.default_rng(4).integers(0, 256, 10_000, dtype=np.uint8).tobytes()
    folded, _ = _spool(tok, data, None, tmp_path)
    out = bytearray()
    with pytest.raises(B.HardShellError) as e:
        B.unfold_pipe_multi([0], tiny_bytes(), tok, _reader(folded[:-100]), out.extend)
    assert e.value.code == B.HS_FORMAT and "truncated block" in str(e.value)
    assert bytes(out) == data[:8192]


def test_pipe_unfold_finds_an_extra_byte_at_the_end(tok):
    container = (GOLDEN / "text_kinds.taco").read_bytes()
    want = (GOLDEN / "text_kinds.in").read_bytes()
    out = bytearray()
    with pytest.raises(B.HardShellError) as e:
        B.unfold_pipe_multi([0], tiny_bytes(), tok, _reader(container + b"\0"), out.extend)
    assert e.value.code == B.HS_FORMAT and "extra bytes" in str(e.value)
    assert bytes(out) == want


def test_pipe_unfold_checks_the_whole_table_before_any_output(tok):
    good = (GOLDEN / "text_kinds.taco").read_bytes()
    cut = good[:C.HEADER_LEN + 5 * 10]  # inside the table
    bad_kind = bytearray(good)
    bad_kind[C.HEADER_LEN + 5 * 16] = 9  # the last entry's kind
    for bad in (good[:50], cut, bytes(bad_kind)):
        out = []
        with pytest.raises(B.HardShellError) as e:
            B.unfold_pipe_multi([0], tiny_bytes(), tok, _reader(bad), out.append)
        assert e.value.code == B.HS_FORMAT
        assert out == []


def test_pipe_unfold_refusals(tok):
    good = (GOLDEN / "text_kinds.taco").read_bytes()

    def bad_read(n):
        raise OSError("gone")

    with pytest.raises(B.HardShellError) as e:
        B.unfold_pipe_multi([0], tiny_bytes(), tok, bad_read, lambda c: None)
    assert e.value.code == B.HS_IO
    # A source that fails after the table: the error is I/O, not a short container.
    pos = [0]

    def fails_late(n):
        if pos[0] > C.HEADER_LEN + 5 * 17:
            raise OSError("gone")
        k = min(n, 7)
        pos[0] += k
        return good[pos[0] - k:pos[0]]

    with pytest.raises(B.HardShellError) as e:
        B.unfold_pipe_multi([0], tiny_bytes(), tok, fails_late, lambda c: None)
    assert e.value.code == B.HS_IO

    def bad_write(chunk):
        raise OSError("disk full")

    with pytest.raises(B.HardShellError) as e:
        B.unfold_pipe_multi([0], tiny_bytes(), tok, _reader(good), bad_write)
    assert e.value.code == B.HS_IO
    # A damaged checksum: HS_CORRUPT after the output.
    bad = bytearray(good)
    bad[50] ^= 1
    with pytest.raises(B.HardShellError) as e:
        _unpipe(tok, bytes(bad))
    assert e.value.code == B.HS_CORRUPT
    # Coded blocks need a GPU: with every GPU refused, the open error.
    coded = (GOLDEN / "predicted_text_k0.taco").read_bytes()
    with pytest.raises(B.HardShellError) as e:
        _unpipe(tok, coded)
    assert e.value.code == B.HS_NO_DEVICE
    assert os.environ["HS_FAIL_OPEN"] == "0,1"


def test_a_length_that_wraps_the_block_count_is_refused(tok):
    """A header whose length needs more blocks than 2^64 bytes can count (2^64 - 1 bytes in blocks
    of 2, block count 0) is a wrong block count, not an empty container of that length."""
    c = C.Container(2, hashlib.sha256(tiny_bytes()).digest(), 2**64 - 1, hashlib.sha256(b"").digest(), 2)
    out = []
    with pytest.raises(B.HardShellError) as e:
        B.unfold_pipe_multi([0], tiny_bytes(), tok, _reader(C.build(c)), out.append)
    assert e.value.code == B.HS_FORMAT and "block count" in str(e.value)
    assert out == []


def test_fold_bound():
    L = B.lib()
    assert L.hs_fold_bound(0, 0) == C.HEADER_LEN
    assert L.hs_fold_bound(1, 0) == C.HEADER_LEN + 5 + 1
    # Block size 0 bounds the spread sizes too: 16 KiB is four blocks of 4 KiB.
    assert L.hs_fold_bound(16384, 0) == C.HEADER_LEN + 5 * 4 + 16384
    assert L.hs_fold_bound(16384, 16384) == C.HEADER_LEN + 5 + 16384
    assert L.hs_fold_bound(2**64 - 1, 1) == 2**64 - 1  # does not fit: saturates


def test_a_version_1_container_reads_as_version_1(tok):
    """conformance/taco-v1-tiny.taco (container version 1, 88-byte header, 5 blocks of 512 bytes)
    was folded with the tiny model of the reference's Rust test builder, not tiny.hsm
    (conformance/README.md). Its header and table read as version 1, so unfolding it with tiny.hsm
    stops at the model check, before any output, as crates/taco/src/unfold.rs checked_model does:
    through a pipe and from memory. A zstd kind in its table (version 2 only) is a format error."""
    data = (GOLDEN / "taco_v1_tiny.taco").read_bytes()
    c = C.parse(data)
    assert c.version == 1 and c.block_size == 512 and c.original_len == 2202
    assert [b.kind for b in c.blocks] == [C.KIND_CODED, C.KIND_CODED, C.KIND_RAW, C.KIND_RAW, C.KIND_CODED]
    out = []
    with pytest.raises(B.HardShellError) as e:
        B.unfold_pipe_multi([0], tiny_bytes(), tok, _reader(data), out.append)
    assert e.value.code == B.HS_MODEL_MISMATCH and out == []
    with pytest.raises(B.HardShellError) as e:
        B.unfold_multi([0], tiny_bytes(), tok, data)
    assert e.value.code == B.HS_MODEL_MISMATCH
    # The third entry (a raw block of 512 bytes) as a zstd block of 10: no such kind in version 1.
    bad = bytearray(data)
    bad[C.HEADER_LEN_V1 + 5 * 2:C.HEADER_LEN_V1 + 5 * 3] = bytes([C.KIND_ZSTD]) + (10).to_bytes(4, "little")
    bad[8:40] = hashlib.sha256(tiny_bytes()).digest()  # past the model check
    with pytest.raises(B.HardShellError) as e:
        B.unfold_pipe_multi([0], tiny_bytes(), tok, _reader(bytes(bad)), out.append)
    assert e.value.code == B.HS_FORMAT and "kind" in str(e.value) and out == []


def test_headers_the_reference_refuses(tok):
    """crates/taco-cli/tests/stream.rs damaged_input_is_an_error...: a header that claims 2^32 - 1
    blocks of 1 byte that the input does not hold is a truncated table (and costs no memory for
    the claimed table), and headers cut at 0, 3, 5, 50 and 103 bytes are format errors."""
    good = (GOLDEN / "text_kinds.taco").read_bytes()
    claims = bytearray(good)
    claims[40:48] = (2**32 - 1).to_bytes(8, "little")
    claims[80:84] = (1).to_bytes(4, "little")
    claims[84:88] = (2**32 - 1).to_bytes(4, "little")
    for data in (bytes(claims), *(good[:n] for n in (0, 3, 5, 50, 103))):
        out = []
        with pytest.raises(B.HardShellError) as e:
            B.unfold_pipe_multi([0], tiny_bytes(), tok, _reader(data), out.append)
        assert e.value.code == B.HS_FORMAT and out == [], len(data)
        assert "truncated" in str(e.value), str(e.value)


def test_an_empty_container_that_names_no_model_unfolds(tok):
    """crates/taco-cli/tests/stream.rs a_raw_only_container_unfolds_without_a_model: the empty
    version 2 container with a zero model hash (block size 65,536) unfolds to nothing, whatever
    the model."""
    c = C.Container(2, bytes(32), 0, hashlib.sha256(b"").digest(), 65536)
    out = bytearray()
    assert B.unfold_pipe_multi([0], tiny_bytes(), tok, _reader(C.build(c)), out.extend) == 0
    assert out == b""
    assert B.unfold_multi([0], tiny_bytes(), tok, C.build(c)) == b""


def _rle_frame(content: int, byte: int) -> bytes:
    """A zstd frame of RLE blocks (RFC 8878 3.1.1.2): a 4-byte content size, then one 4-byte
    block of `byte` for each 128 KiB."""
    f = bytearray([0x28, 0xB5, 0x2F, 0xFD, 0x80, 10 << 3]) + content.to_bytes(4, "little")
    left = content
    while left > 0:
        n = min(left, 128 * 1024)
        left -= n
        f += ((1 if left == 0 else 0) | (1 << 1) | (n << 3)).to_bytes(4, "little")[:3] + bytes([byte])
    return bytes(f)


@pytest.mark.parametrize("content", [4096, 3900])
def test_a_zstd_frame_that_does_not_give_its_block_is_a_format_error(tok, content):
    """crates/taco/tests/security_unfold.rs zstd_frame_longer_than_its_block_is_refused: a block
    of 4,000 bytes whose frame states another length is FormatError::CorruptZstdBlock, in memory
    and through a pipe."""
    c = C.Container(2, bytes(32), 4000, hashlib.sha256(b"A" * 4000).digest(), 4000)
    c.blocks = [C.Block(0, C.KIND_ZSTD, 4000, _rle_frame(content, ord("A")))]
    data = C.build(c)
    with pytest.raises(B.HardShellError) as e:
        B.unfold_multi([0], tiny_bytes(), tok, data)
    assert e.value.code == B.HS_FORMAT and "CorruptZstdBlock" in str(e.value)
    out = []
    with pytest.raises(B.HardShellError) as e:
        B.unfold_pipe_multi([0], tiny_bytes(), tok, _reader(data), out.append)
    assert e.value.code == B.HS_FORMAT and out == []
    # The frame of the right length gives the block.
    c.blocks = [C.Block(0, C.KIND_ZSTD, 4000, _rle_frame(4000, ord("A")))]
    assert B.unfold_multi([0], tiny_bytes(), tok, C.build(c)) == b"A" * 4000


@pytest.mark.parametrize("name", NO_CODED)
def test_seekable_unfold_on_worker_threads_gives_the_published_input(tok, name):
    """hs_unfold_stream_multi: the containers without coded blocks, read by offset."""
    container = (GOLDEN / (name + ".taco")).read_bytes()
    out = bytearray()
    n = B.unfold_stream_multi([0], tiny_bytes(), tok, len(container), lambda at, k: container[at:at + k], out.extend)
    assert n == len(out) and bytes(out) == (GOLDEN / (name + ".in")).read_bytes()
    # A container one byte short: refused before any output (the length is checked first).
    out2 = []
    with pytest.raises(B.HardShellError) as e:
        B.unfold_stream_multi([0], tiny_bytes(), tok, len(container) - 1, lambda at, k: container[at:at + k],
                              out2.append)
    assert e.value.code == B.HS_FORMAT and out2 == []


def test_one_batch_wrappers_reach_the_library(tok):
    """The Python wrappers of the one-batch entry points run only on a GPU otherwise. With a null
    batch handle each must reach its C function with the right arguments and come back with the
    library's refusal of the null argument."""
    import types

    nobatch = types.SimpleNamespace(h=None)
    data = b"some text"
    container = (GOLDEN / "one_byte.taco").read_bytes()
    calls = [
        lambda: B.fold(nobatch, tok, data),
        lambda: B.fold_stream(nobatch, tok, len(data), _reader(data), lambda at, c: None),
        lambda: B.fold_spool(nobatch, tok, _reader(data), lambda c: None),
        lambda: B.fold_spool(nobatch, tok, _reader(data), lambda c: None, length=len(data)),
        lambda: B.unfold(nobatch, tok, container),
        lambda: B.unfold_stream(nobatch, tok, len(container), lambda at, k: container[at:at + k], lambda c: None),
        lambda: B.unfold_pipe(nobatch, tok, _reader(container), lambda c: None),
    ]
    for i, call in enumerate(calls):
        with pytest.raises(B.HardShellError) as e:
            call()
        assert e.value.code == B.HS_BAD_ARGUMENT and "null" in str(e.value), (i, e.value)


@pytest.mark.parametrize("size", [0, 1, 4097, 9000])
def test_seekable_outputs_place_blocks_table_and_header(tok, size):
    """The seekable layouts (stream.rs SeekLayout): hs_fold_multi into memory and
    hs_fold_stream_multi into a callback at offsets give the container of the spool method, with
    the header at 0, the table after it and the blocks after the table, across segments."""
    data = np.random.default_rng(size + 1).integers(0, 256, size, dtype=np.uint8).tobytes()
    want = _raw_container(data)
    got, stats = B.fold_multi([0], tiny_bytes(), tok, data, block_size=1)
    assert got == want and stats["blocks"] == size
    buf = bytearray()

    def write_at(at, chunk):
        if len(buf) < at + len(chunk):
            buf.extend(bytes(at + len(chunk) - len(buf)))
        buf[at:at + len(chunk)] = chunk

    n, _ = B.fold_stream_multi([0], tiny_bytes(), tok, size, _reader(data), write_at, 1, 0)
    assert n == len(want) and bytes(buf) == want
    # An output one byte too small for hs_fold_multi: refused with the length it needs.
    cap = np.zeros(max(len(want) - 1, 1), np.uint8)
    m = ctypes.c_size_t()
    opt = B.FoldOptions(1, 0, 0, 0)
    ords = np.zeros(1, np.int32)
    rc = B.lib().hs_fold_multi(ords.ctypes.data, 1, tiny_bytes(), len(tiny_bytes()), 256, 16384, tok.h, data,
                               len(data), ctypes.byref(opt), cap.ctypes.data, len(want) - 1, ctypes.byref(m), None)
    assert rc == B.HS_BAD_ARGUMENT and m.value == len(want)
