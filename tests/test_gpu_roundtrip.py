"""Round-trip correctness at GPT-2 scale: the CPU oracle and one B200 give
the same intervals and the same `.taco` bytes (so the same SHA-256).

The model is the synthetic GPT-2 124M `.hsm` (12 layers, d 768, vocabulary 50,257, context
1,024). The GPU side is `hs_fold` (tokenizer, zstd, the coder op on the GPU, the range encoder,
the container). The CPU side builds the container from the oracle alone: the oracle's fast path
gives every interval (one slot, the context restarting as the reference session does), the
oracle's range encoder codes them with the stop rule of crates/taco/src/codec.rs:70-131, and
the block takes its smallest form, with the header of crates/taco-format. Both sides tokenize
with the product tokenizer, which is pinned on its own (tests/test_tokenizer.py).

Two inputs: 3,672 bytes of seeded Zipf text over 5,000 lowercase words (the config), and 1,000
bytes that the model itself predicts (each byte the model's most likely single-byte token). With
random-init weights the model spends about 15.6 bits on a token, so zstd wins both blocks: the
comparison covers every interval, the encoder up to its stop rule, and the container. The bytes
of winning coded blocks are pinned by the conformance vectors of the tiny model
(tests/test_gpu_fold.py). Then the container unfolds on the GPU to the input.
"""

import ctypes
import hashlib

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import container as C
from taco_b200 import synth

pytestmark = pytest.mark.gpu


def _zstd(data: bytes) -> bytes:
    """One zstd frame at level 19, content size, no checksum, no dictionary id (zstd_block.rs)."""
    z = ctypes.CDLL("libzstd.so.1")
    z.ZSTD_createCCtx.restype = ctypes.c_void_p
    z.ZSTD_freeCCtx.argtypes = [ctypes.c_void_p]
    z.ZSTD_CCtx_setParameter.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    z.ZSTD_CCtx_setParameter.restype = ctypes.c_size_t
    z.ZSTD_compressBound.argtypes = [ctypes.c_size_t]
    z.ZSTD_compressBound.restype = ctypes.c_size_t
    z.ZSTD_compress2.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t]
    z.ZSTD_compress2.restype = ctypes.c_size_t
    cctx = z.ZSTD_createCCtx()
    for p, v in ((100, 19), (200, 1), (201, 0), (202, 0)):
        z.ZSTD_CCtx_setParameter(cctx, p, v)
    cap = z.ZSTD_compressBound(len(data))
    buf = ctypes.create_string_buffer(cap)
    n = z.ZSTD_compress2(cctx, buf, cap, data, len(data))
    z.ZSTD_freeCCtx(cctx)
    return buf.raw[:n]


def _varint(v: int) -> bytes:
    out = bytearray()
    while v >= 0x80:
        out.append((v & 0x7F) | 0x80)
        v >>= 7
    out.append(v)
    return bytes(out)


def _cpu_container(om, model_bytes, tokens, data, eot, vocab):
    """The container of `data` (one block of the default 16 KiB) from the oracle alone, and the
    oracle's intervals."""
    n = len(tokens)
    fast = O.FastBatch(om, 1, 0)
    inputs = [eot] + [int(t) for t in tokens[:-1]]
    iv = fast.run_coded([0] * n, inputs, [0] * n, [int(t) for t in tokens], 32)
    zframe = _zstd(data)
    stop = min(len(data), len(zframe))
    prefix = len(_varint(n))
    coded = None
    if prefix < stop:
        enc = O.Encoder()
        live = True
        for sym, start, freq in iv:
            enc.interval(int(start), int(freq), int(sym) == vocab - 1, 32)
            if prefix + enc.min_final_len() >= stop:
                live = False
                break
        if live:
            coded = _varint(n) + enc.finish()
    kind, stored = C.KIND_RAW, data
    if len(zframe) < len(stored):
        kind, stored = C.KIND_ZSTD, zframe
    if coded is not None and len(coded) < len(stored):
        kind, stored = C.KIND_CODED, coded
    c = C.Container(2, hashlib.sha256(model_bytes).digest(), len(data), hashlib.sha256(data).digest(), 16384)
    c.blocks = [C.Block(0, kind, len(data), stored)]
    return C.build(c), iv


@pytest.fixture(scope="module")
def gpt2():
    model_bytes = synth.gpt2_hsm(124)
    dev = B.CudaDevice(0)
    model = B.CudaModel(dev, model_bytes)
    batch = B.CudaBatch(model, 4, 4096)
    tok = B.Tokenizer(model_bytes)
    om = O.Model(model_bytes)
    yield model_bytes, model, batch, tok, om
    tok.close()
    batch.close()
    model.close()
    dev.close()


def _check(gpt2, data):
    model_bytes, model, batch, tok, om = gpt2
    eot, vocab = model.eot_token(), model.vocab_size()
    tokens = tok.encode(data)
    want, iv_cpu = _cpu_container(om, model_bytes, tokens, data, eot, vocab)
    # The intervals of the GPU equal the oracle's, row for row.
    batch.reset(0)
    inputs = np.concatenate([[eot], tokens[:-1]]).astype(np.uint32)
    got_iv = batch.run_coded(np.zeros(len(tokens)), inputs, np.zeros(len(tokens)), tokens, 32)
    assert np.array_equal(np.stack([got_iv["symbol"], got_iv["start"], got_iv["freq"]], 1).astype(np.uint64),
                          np.asarray(iv_cpu, dtype=np.uint64))
    got, stats = B.fold(batch, tok, data)
    assert hashlib.sha256(got).hexdigest() == hashlib.sha256(want).hexdigest()
    assert stats["tokens"] == len(tokens)
    assert B.unfold(batch, tok, got) == data


def test_zipf_text_gives_the_oracles_container(gpt2):
    data = synth.zipf_text(3672, seed=3672)[:3672]
    assert len(data) == 3672
    _check(gpt2, data)


def test_model_predicted_bytes_give_the_oracles_container(gpt2):
    model_bytes, model, batch, tok, om = gpt2
    eot = model.eot_token()
    # Each next byte is the model's most likely single-byte token after the bytes so far.
    batch.reset(1)
    out, prev = [], eot
    for _ in range(1000):
        w = batch.run_weights([1], [prev])[0]
        prev = int(np.argmax(w[:256]))
        out.append(prev)
    _check(gpt2, bytes(out))
