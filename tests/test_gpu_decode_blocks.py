"""hs_batch_decode_blocks, the unfold of coded blocks with the range decoder on the device,
against the published containers and the CPU oracle (needs a B200).

- The coded blocks of the three conformance containers decode, all blocks of a container in one
  call (one slot each), to the container's input bytes (crates/taco/src/codec.rs BlockDecoder).
- Synthetic blocks on a model with 64-wide heads (the decode attention and the staged values
  cache): the oracle codes random token streams (its fast path's Encode intervals and its range
  encoder); the device decodes them back, including blocks longer than the context (restart
  steps with an overlap), blocks of one token and an empty block. The slot positions after the
  call equal the oracle's.
- Validation: two blocks in one slot, more blocks than max_rows, freq_bits out of range.
"""

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import container as C
from taco_b200 import synth

from .common import GOLDEN, tiny_bytes

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    d = B.CudaDevice(0)
    yield d
    d.close()


def _split(payload: bytes):
    """codec.rs: a coded block is the varint token count, then the range coder's bytes."""
    end = next(i for i, byte in enumerate(payload) if byte < 0x80) + 1
    count = 0
    for i, byte in enumerate(payload[:end]):
        count |= (byte & 0x7F) << (7 * i)
    return count, payload[end:]


@pytest.mark.parametrize("name", ["predicted_text_k0", "predicted_text_k32", "all_kinds_text"])
def test_conformance_blocks_decode_on_the_device(dev, name):
    om = O.Model(tiny_bytes())
    model = B.CudaModel(dev, tiny_bytes())
    c = C.parse((GOLDEN / (name + ".taco")).read_bytes())
    coded = [b for b in c.blocks if b.kind == C.KIND_CODED]
    assert coded
    batch = B.CudaBatch(model, len(coded), 64)
    batch.set_overlap(c.overlap)
    counts, payloads = zip(*(_split(b.stored) for b in coded))
    toks, status = batch.decode_blocks(list(range(len(coded))), list(payloads), list(counts), 32)
    assert not status.any()
    decoded = {id(b): b"".join(om.token_bytes(int(t)) for t in tk) for b, tk in zip(coded, toks)}
    out = bytearray()
    for b in c.blocks:
        if b.kind == C.KIND_RAW:
            out += b.stored
        elif b.kind == C.KIND_ZSTD:
            out += C.decode_zstd(b.stored, b.original_len)
        else:
            assert len(decoded[id(b)]) == b.original_len
            out += decoded[id(b)]
    assert bytes(out) == (GOLDEN / (name + ".in")).read_bytes()
    batch.close()
    model.close()


def _encode_streams(om, streams, overlap, bits):
    """The oracle's coding of each token stream from a fresh slot: the Encode interval of every
    token after the inputs EOT, t0, t1, ..., then the range encoder."""
    n = len(streams)
    fast = O.FastBatch(om, n, overlap)
    longest = max(len(s) for s in streams)
    enc = [O.Encoder() for _ in range(n)]
    for j in range(longest):
        live = [i for i in range(n) if len(streams[i]) > j]
        inputs = [om.eot if j == 0 else int(streams[i][j - 1]) for i in live]
        toks = [int(streams[i][j]) for i in live]
        iv = fast.run_coded(live, inputs, [0] * len(live), toks, bits)
        for k, i in enumerate(live):
            sym, start, freq = (int(x) for x in iv[k])
            assert sym == toks[k]
            enc[i].interval(start, freq, sym == om.vocab - 1, bits)
    return [e.finish() for e in enc], [fast.position(i) for i in range(n)]


@pytest.mark.parametrize("bits", [32, 24])
def test_synthetic_blocks_round_trip_through_the_device_decoder(dev, bits):
    data = synth.gpt2_hsm(7, shape=synth.MINI)
    om = O.Model(data)
    model = B.CudaModel(dev, data)
    rng = np.random.default_rng(bits)
    lens = [700, 1, 513, 0, 40] + rng.integers(2, 300, 27).tolist()  # 700, 513: past n_ctx = 512
    streams = [rng.integers(0, om.vocab, n).astype(np.uint32) for n in lens]
    overlap = 20
    payloads, positions = _encode_streams(om, streams, overlap, bits)
    batch = B.CudaBatch(model, len(streams) + 3, 256)
    batch.set_overlap(overlap)
    slots = [s + 3 for s in range(len(streams))]  # not in slot order 0..n-1
    toks, status = batch.decode_blocks(slots, payloads, lens, bits)
    assert not status.any()
    for i, s in enumerate(streams):
        assert np.array_equal(toks[i], s), i
        assert batch.position(slots[i]) == positions[i], i
    batch.close()
    model.close()


def test_decode_blocks_refuses_bad_calls(dev):
    model = B.CudaModel(dev, tiny_bytes())
    batch = B.CudaBatch(model, 4, 2)
    with pytest.raises(B.HardShellError) as e:
        batch.decode_blocks([1, 1], [b"\x00", b"\x00"], [1, 1], 32)
    assert e.value.code == B.HS_BAD_ARGUMENT
    with pytest.raises(B.HardShellError) as e:
        batch.decode_blocks([0, 1, 2], [b"", b"", b""], [1, 1, 1], 32)
    assert e.value.code == B.HS_UNSUPPORTED
    with pytest.raises(B.HardShellError) as e:
        batch.decode_blocks([0], [b""], [1], 8)  # 2^8 < vocab 300
    assert e.value.code == B.HS_UNSUPPORTED
    with pytest.raises(B.HardShellError) as e:
        batch.decode_blocks([9], [b""], [1], 32)
    assert e.value.code == B.HS_BAD_SLOT
    batch.close()
    model.close()
