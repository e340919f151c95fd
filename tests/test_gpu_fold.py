"""The fold of the profile text (hs_fold: tokenizer, zstd, the coder op on the GPU, the range
encoder with its stop rule, the container writer) on a B200, against the published containers.

Every text-profile conformance input folds with the vector's block size and overlap
(vectors.tsv) and the tiny model. The container must equal the published bytes, except where the
zstd library of this image (1.5.5) writes another frame than the reference's pinned 1.5.7: such
a block must be the only difference, must decode to its bytes, and the header and every other
block must be equal. The vectors whose zstd frames agree (and those without zstd blocks) must be
equal byte for byte. A larger input of mixed text and binary folds and every block decodes.
"""

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import container as C

from .common import GOLDEN, tiny_bytes

TEXT_VECTORS = ["empty", "one_byte", "random_raw", "text_k0", "text_k20", "text_kinds",
                "predicted_text_k0", "predicted_text_k32", "all_kinds_text"]
EXACT = {"empty", "one_byte", "random_raw", "text_k0", "text_k20", "predicted_text_k0", "predicted_text_k32"}

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup():
    dev = B.CudaDevice(0)
    model = B.CudaModel(dev, tiny_bytes())
    batch = B.CudaBatch(model, 8, 4096)
    tok = B.Tokenizer(tiny_bytes())
    yield batch, tok
    tok.close()
    batch.close()
    model.close()
    dev.close()


def _vector(name):
    for line in (GOLDEN / "vectors.tsv").read_text().splitlines():
        f = line.split("\t")
        if f[0] == name:
            return (0 if f[2] == "default" else int(f[2])), (0 if f[3] == "default" else int(f[3]))
    raise KeyError(name)


def _decode(om, c, b):
    if b.kind == C.KIND_RAW:
        return b.stored
    if b.kind == C.KIND_ZSTD:
        return C.decode_zstd(b.stored, b.original_len)
    data, _ = O.decode_block(om, b.stored, b.original_len, c.overlap)
    return data


@pytest.mark.parametrize("name", TEXT_VECTORS)
def test_fold_gives_the_published_container(setup, name):
    batch, tok = setup
    om = O.Model(tiny_bytes())
    bs, k = _vector(name)
    data = (GOLDEN / (name + ".in")).read_bytes()
    want = (GOLDEN / (name + ".taco")).read_bytes()
    got, stats = B.fold(batch, tok, data, bs, k)
    assert stats["original_len"] == len(data) and stats["container_len"] == len(got)
    if name in EXACT:
        assert got == want
        return
    if got == want:
        return
    g, w = C.parse(got), C.parse(want)
    for f in ("version", "model_hash", "original_len", "checksum", "block_size", "profile", "overlap"):
        assert getattr(g, f) == getattr(w, f), f
    off = 0
    for gb, wb in zip(g.blocks, w.blocks, strict=True):
        orig = data[off:off + gb.original_len]
        off += gb.original_len
        if (gb.kind, gb.stored) != (wb.kind, wb.stored):
            assert C.KIND_ZSTD in (gb.kind, wb.kind), gb.index  # a zstd frame of another version
        assert _decode(om, g, gb) == orig


def test_a_larger_input_folds_and_every_block_decodes(setup):
    batch, tok = setup
    om = O.Model(tiny_bytes())
    rng = np.random.default_rng(11)
    # Model-predicted text (coded blocks win there), binary bytes, mixed text, ill-formed UTF-8.
    pred = (GOLDEN / "predicted_text_k0.in").read_bytes()
    data = pred + rng.integers(0, 256, 700, dtype=np.uint8).tobytes() + \
        (GOLDEN / "all_kinds_text.in").read_bytes() + pred + "ünï ✓".encode() + b"\xff\xfe"
    for bs, k, coded in [(300, 0, True), (300, 16, True), (777, 12, False), (0, 0, False)]:
        got, stats = B.fold(batch, tok, data, bs, k, threads=4)
        c = C.parse(got)
        assert c.original_len == len(data) and c.overlap == k
        assert stats["blocks"] == len(c.blocks)
        assert stats["coded_blocks"] == sum(b.kind == C.KIND_CODED for b in c.blocks)
        if coded:
            assert stats["coded_blocks"] > 0
        out = b"".join(_decode(om, c, b) for b in c.blocks)
        assert out == data


@pytest.mark.parametrize("name", TEXT_VECTORS)
def test_unfold_gives_the_published_inputs(setup, name):
    batch, tok = setup
    want = (GOLDEN / (name + ".in")).read_bytes()
    assert B.unfold(batch, tok, (GOLDEN / (name + ".taco")).read_bytes()) == want


def test_fold_then_unfold_round_trips(setup):
    batch, tok = setup
    rng = np.random.default_rng(12)
    pred = (GOLDEN / "predicted_text_k32.in").read_bytes()
    data = pred * 3 + rng.integers(0, 256, 333, dtype=np.uint8).tobytes() + pred
    for bs, k in [(300, 32), (64, 0), (5000, 7)]:
        got, stats = B.fold(batch, tok, data, bs, k)
        assert B.unfold(batch, tok, got) == data


def test_unfold_refuses_bad_containers(setup):
    batch, tok = setup
    good = (GOLDEN / "all_kinds_text.taco").read_bytes()

    def code(blob):
        with pytest.raises(B.HardShellError) as e:
            B.unfold(batch, tok, blob, original_len=1 << 16)
        return e.value.code

    assert code(b"TACX" + good[4:]) == B.HS_FORMAT
    assert code(good[:-1]) == B.HS_FORMAT
    assert code(good + b"\0") == B.HS_FORMAT
    c = C.parse(good)
    other = bytearray(good)
    other[8] ^= 1  # another model's hash
    assert code(bytes(other)) == B.HS_MODEL_MISMATCH
    wrong_sum = bytearray(good)
    wrong_sum[48] ^= 1
    assert code(bytes(wrong_sum)) == B.HS_CORRUPT
    # A damaged coded block: its tokens no longer give its bytes (or an interval misses).
    coded = next(b for b in c.blocks if b.kind == C.KIND_CODED)
    c2 = C.parse(good)
    blk = c2.blocks[coded.index]
    blk.stored = blk.stored[:2] + bytes(x ^ 0x5A for x in blk.stored[2:])
    assert code(C.build(c2)) == B.HS_CORRUPT
    # A mixed block (profile logs) needs the caller's mixer.
    c3 = C.parse(good)
    c3.profile, c3.mixer_rule = C.PROFILE_LOGS, 1
    c3.blocks[coded.index].kind = C.KIND_MIXED
    assert code(C.build(c3)) == B.HS_UNSUPPORTED


def test_fold_on_several_gpu_threads_equals_one_gpu(setup):
    """hs_fold_multi deals the windows to one host thread per GPU; the container is hs_fold's. On
    a box with one GPU both threads use device 0 (two handles, two batches)."""
    batch, tok = setup
    import torch

    ords = [0, 1] if torch.cuda.device_count() >= 2 else [0, 0]
    pred = (GOLDEN / "predicted_text_k32.in").read_bytes()
    data = pred * 4 + (GOLDEN / "all_kinds_text.in").read_bytes()
    for bs, k in [(300, 32), (2000, 5)]:
        want, _ = B.fold(batch, tok, data, bs, k)
        got, stats = B.fold_multi(ords, tiny_bytes(), tok, data, bs, k, slots=8, max_rows=4096)
        assert got == want
        assert stats["coded_blocks"] > 0 or bs == 2000
    assert stats["gpus_failed"] == 0


def test_fold_moves_the_windows_of_a_gpu_that_fails_to_open(setup, monkeypatch):
    """A GPU whose open fails (HS_FAIL_OPEN refuses it on the host, no GPU fault) gives its windows
    to the others: the container is still hs_fold's, and the stats count the failed GPU. With every
    GPU refused, the fold fails with the open's error."""
    batch, tok = setup
    data = (GOLDEN / "predicted_text_k32.in").read_bytes() * 3
    want, _ = B.fold(batch, tok, data, 300, 32)
    monkeypatch.setenv("HS_FAIL_OPEN", "7")
    got, stats = B.fold_multi([0, 7, 0], tiny_bytes(), tok, data, 300, 32, slots=8, max_rows=4096)
    assert got == want
    assert stats["gpus_failed"] == 1
    monkeypatch.setenv("HS_FAIL_OPEN", "0,7")
    with pytest.raises(B.HardShellError) as e:
        B.fold_multi([0, 7], tiny_bytes(), tok, data, 300, 32, slots=8, max_rows=4096)
    assert e.value.code == B.HS_NO_DEVICE


# ---- streams: the same bytes segment by segment, bounded memory (crates/taco/src/stream.rs) ----

def _reader(data: bytes):
    pos = [0]

    def read(n):
        out = data[pos[0]:pos[0] + n]
        pos[0] += len(out)
        return out

    return read


def _seekable():
    buf = bytearray()

    def write(at, chunk):
        if len(buf) < at + len(chunk):
            buf.extend(bytes(at + len(chunk) - len(buf)))
        buf[at:at + len(chunk)] = chunk

    return buf, write


def _many_blocks():
    """More than one segment (4,096 blocks) of 256-byte blocks: coded, zstd and raw blocks."""
    pred = (GOLDEN / "predicted_text_k32.in").read_bytes()
    rng = np.random.default_rng(17)
    parts = [pred, rng.integers(0, 256, 40_000, dtype=np.uint8).tobytes(), (GOLDEN / "all_kinds_text.in").read_bytes()]
    data = b""
    while len(data) < 4100 * 256 + 77:
        data += parts[len(data) % 3]
    return data[:4100 * 256 + 77]


@pytest.mark.parametrize("case", ["vector", "segments"])
def test_fold_stream_gives_the_bytes_of_fold(setup, case):
    batch, tok = setup
    if case == "vector":
        data, bs, k = (GOLDEN / "predicted_text_k32.in").read_bytes() * 2, 300, 32
    else:
        data, bs, k = _many_blocks(), 256, 5
    want, wstats = B.fold(batch, tok, data, bs, k)
    buf, write = _seekable()
    n, stats = B.fold_stream(batch, tok, len(data), _reader(data), write, bs, k)
    assert n == len(want) and bytes(buf) == want
    for key in ("blocks", "coded_blocks", "zstd_blocks", "tokens", "container_len"):
        assert stats[key] == wstats[key]
    assert stats["coded_blocks"] > 0
    # The unfold stream gives the input back.
    out = bytearray()
    got_len = B.unfold_stream(batch, tok, len(want), lambda at, m: want[at:at + m], out.extend)
    assert got_len == len(data) and bytes(out) == data
    if case == "segments":
        ords = [0, 1] if __import__("torch").cuda.device_count() >= 2 else [0, 0]
        buf2, write2 = _seekable()
        n2, _ = B.fold_stream_multi(ords, tiny_bytes(), tok, len(data), _reader(data), write2, bs, k, slots=8,
                                    max_rows=4096)
        assert bytes(buf2) == want


@pytest.mark.parametrize("known", [True, False])
def test_spool_fold_and_pipe_unfold_give_the_bytes_of_fold(setup, tmp_path, known):
    """hs_fold_spool (StreamFold::to_writer) gives the container of hs_fold, with the input length
    known or not, across segments with coded, zstd and raw blocks; hs_unfold_pipe
    (StreamUnfold::from_reader) gives the input back from the container read in one pass."""
    batch, tok = setup
    data, bs, k = _many_blocks(), 256, 5
    want, wstats = B.fold(batch, tok, data, bs, k)
    out = bytearray()
    n, stats = B.fold_spool(batch, tok, _reader(data), out.extend, len(data) if known else None, tmp_path, bs, k)
    assert n == len(want) and bytes(out) == want
    for key in ("blocks", "coded_blocks", "zstd_blocks", "tokens", "container_len", "original_len"):
        assert stats[key] == wstats[key]
    assert stats["coded_blocks"] > 0 and list(tmp_path.iterdir()) == []
    restored = bytearray()
    assert B.unfold_pipe(batch, tok, _reader(want), restored.extend) == len(data)
    assert bytes(restored) == data
    if not known:
        # Two GPUs when there are two, else the two worker threads of one (as the unfold test
        # on several GPU threads below).
        ords = [0, 1] if __import__("torch").cuda.device_count() >= 2 else [0]
        out2 = bytearray()
        B.fold_spool_multi(ords, tiny_bytes(), tok, _reader(data), out2.extend, None, tmp_path, bs, k, slots=8,
                           max_rows=4096)
        assert bytes(out2) == want
        restored2 = bytearray()
        B.unfold_pipe_multi(ords, tiny_bytes(), tok, _reader(want), restored2.extend, slots=8, max_rows=4096)
        assert bytes(restored2) == data


def test_pipe_unfold_gives_the_published_inputs(setup):
    batch, tok = setup
    for name in TEXT_VECTORS:
        container = (GOLDEN / (name + ".taco")).read_bytes()
        out = bytearray()
        B.unfold_pipe(batch, tok, _reader(container), out.extend)
        assert bytes(out) == (GOLDEN / (name + ".in")).read_bytes()
    # A missing byte inside a coded block, and an extra byte after the last.
    good = (GOLDEN / "predicted_text_k32.taco").read_bytes()
    for bad, why in ((good[:-1], "truncated block"), (good + b"\0", "extra bytes")):
        with pytest.raises(B.HardShellError) as e:
            B.unfold_pipe(batch, tok, _reader(bad), lambda c: None)
        assert e.value.code == B.HS_FORMAT and why in str(e.value)


def test_fold_stream_refuses_a_short_or_long_source_and_a_failing_sink(setup):
    batch, tok = setup
    data = (GOLDEN / "predicted_text_k32.in").read_bytes()
    for length in (len(data) + 1, len(data) - 1):
        _, write = _seekable()
        with pytest.raises(B.HardShellError) as e:
            B.fold_stream(batch, tok, length, _reader(data), write, 300, 0)
        assert e.value.code == B.HS_IO

    def bad_write(at, chunk):
        raise OSError("disk full")

    with pytest.raises(B.HardShellError) as e:
        B.fold_stream(batch, tok, len(data), _reader(data), bad_write, 300, 0)
    assert e.value.code == B.HS_IO


def test_unfold_stream_refuses_a_damaged_table_before_any_output(setup):
    batch, tok = setup
    good = (GOLDEN / "predicted_text_k32.taco").read_bytes()
    for bad in (good[:-1], good + b"\0", good[:150]):
        out = []
        with pytest.raises(B.HardShellError) as e:
            B.unfold_stream(batch, tok, len(bad), lambda at, m, d=bad: d[at:at + m], out.append)
        assert e.value.code == B.HS_FORMAT
        assert out == []


def test_unfold_on_several_gpu_threads_equals_one_gpu(setup):
    """hs_unfold_multi deals each segment's coded blocks to worker threads (two per GPU); the
    output is hs_unfold's, and a damaged coded block is reported as by hs_unfold."""
    batch, tok = setup
    import torch

    ords = [0, 1] if torch.cuda.device_count() >= 2 else [0]
    for name in ["predicted_text_k0", "predicted_text_k32", "all_kinds_text"]:
        c = (GOLDEN / (name + ".taco")).read_bytes()
        want = (GOLDEN / (name + ".in")).read_bytes()
        assert B.unfold_multi(ords, tiny_bytes(), tok, c, slots=8, max_rows=4096) == want
    # Many coded blocks in many rounds: a fold of the predicted text in 300-byte blocks.
    data = (GOLDEN / "predicted_text_k32.in").read_bytes() * 6
    folded, stats = B.fold(batch, tok, data, 300, 32)
    assert stats["coded_blocks"] > 8
    assert B.unfold_multi(ords, tiny_bytes(), tok, folded, slots=4, max_rows=4096) == data
    cont = C.parse(folded)
    coded = [b for b in cont.blocks if b.kind == C.KIND_CODED]
    blk = cont.blocks[coded[3].index]
    blk.stored = blk.stored[:2] + bytes(x ^ 0x5A for x in blk.stored[2:])
    with pytest.raises(B.HardShellError) as e:
        B.unfold_multi(ords, tiny_bytes(), tok, C.build(cont), slots=4, max_rows=4096)
    assert e.value.code == B.HS_CORRUPT
