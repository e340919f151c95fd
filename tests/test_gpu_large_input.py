"""The large mixed input of BASELINE configs[4] (Zipf text, JSON-shaped key/number records and
uniform random bytes in 64 KiB pieces, taco_b200/synth.py mixed_stream) on the synthetic GPT-2
124M model, at a reduced size: one piece of each kind, 12 blocks of the default 16 KiB.

- hs_fold on one GPU, hs_fold_multi over two GPU threads and hs_fold_stream give the same
  container.
- Every block is stored as the CPU path stores it. The CPU path is the oracle alone: one slot per
  block, the context restarting as the reference session does, the oracle's intervals run window
  by window into its range encoder with the stop rule of crates/taco/src/codec.rs:70-131, zstd
  level 19, and the smallest form (writer.rs:89). Tokens come from the product tokenizer, which
  is pinned on its own (tests/test_tokenizer.py).
- The container unfolds to the input.

The full 256 MiB stream runs in bench.py (`large_input`), where its SHA-256 at every GPU count is
reported; the CPU path there is out of reach (about 10^8 tokens at about 2 K tokens/s).
"""

import hashlib
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import container as C
from taco_b200 import synth

from .test_gpu_roundtrip import _varint, _zstd

pytestmark = pytest.mark.gpu

PIECE = 64 << 10
BLOCK = 16 << 10


def _sample() -> bytes:
    """The first piece of each kind of a 2 MiB mixed stream, in stream order."""
    n = 32
    kinds = synth.mixed_kinds(n)
    data = synth.mixed_stream(n * PIECE)
    out, seen = [], set()
    for i, k in enumerate(kinds.tolist()):
        if k not in seen:
            seen.add(k)
            out.append(data[i * PIECE:(i + 1) * PIECE])
    assert seen == {0, 1, 2}
    return b"".join(out)


def _cpu_block(om, tokens, data, eot, vocab, window=1023):
    """(kind, stored bytes) of one block by the CPU path; the oracle runs the block's inputs a window
    at a time and stops when the encoder stops."""
    n = len(tokens)
    zframe = _zstd(data)
    stop = min(len(data), len(zframe))
    prefix = len(_varint(n))
    coded = None
    if n and prefix < stop:
        fast = O.FastBatch(om, 1, 0)
        inputs = np.concatenate([[eot], tokens[:-1]]).astype(np.uint32)
        enc = O.Encoder()
        live = True
        for s0 in range(0, n, window):
            s1 = min(n, s0 + window)
            iv = fast.run_coded(np.zeros(s1 - s0, np.uint32), inputs[s0:s1], np.zeros(s1 - s0, np.uint32),
                                tokens[s0:s1].astype(np.uint64), 32, threads=1)
            for sym, start, freq in iv:
                enc.interval(int(start), int(freq), int(sym) == vocab - 1, 32)
                if prefix + enc.min_final_len() >= stop:
                    live = False
                    break
            if not live:
                break
        if live:
            coded = _varint(n) + enc.finish()
    kind, stored = C.KIND_RAW, data
    if len(zframe) < len(stored):
        kind, stored = C.KIND_ZSTD, zframe
    if coded is not None and len(coded) < len(stored):
        kind, stored = C.KIND_CODED, coded
    return kind, stored


def test_mixed_input_sample_equals_the_cpu_path_block_by_block():
    import torch

    model_bytes = synth.gpt2_hsm(124)
    data = _sample()
    dev = B.CudaDevice(0)
    model = B.CudaModel(dev, model_bytes)
    batch = B.CudaBatch(model, 64, 16384)
    tok = B.Tokenizer(model_bytes)
    try:
        got, stats = B.fold(batch, tok, data)
        assert stats["blocks"] == len(data) // BLOCK
        assert stats["gpu_rows"] > 0
        ords = [0, 1] if torch.cuda.device_count() >= 2 else [0, 0]
        multi, _ = B.fold_multi(ords, model_bytes, tok, data, slots=64, max_rows=16384)
        assert multi == got
        buf = bytearray(len(got))

        def write(at, chunk):
            buf[at:at + len(chunk)] = chunk

        pos = [0]

        def read(n):
            out = data[pos[0]:pos[0] + n]
            pos[0] += len(out)
            return out

        n, _ = B.fold_stream(batch, tok, len(data), read, write)
        assert bytes(buf[:n]) == got
        assert B.unfold(batch, tok, got) == data
        eot, vocab = model.eot_token(), model.vocab_size()
        c = C.parse(got)
    finally:
        tok_bytes = [tok.encode(data[i:i + BLOCK]) for i in range(0, len(data), BLOCK)]
        tok.close()
        batch.close()
        model.close()
        dev.close()
    om = O.Model(model_bytes)
    with ThreadPoolExecutor(max_workers=len(tok_bytes)) as ex:
        want = list(ex.map(lambda i: _cpu_block(om, tok_bytes[i], data[i * BLOCK:(i + 1) * BLOCK], eot, vocab),
                           range(len(tok_bytes))))
    for i, (b, (kind, stored)) in enumerate(zip(c.blocks, want)):
        assert (b.kind, b.stored) == (kind, stored), i
    cpu = C.Container(2, hashlib.sha256(model_bytes).digest(), len(data), hashlib.sha256(data).digest(), BLOCK)
    cpu.blocks = [C.Block(i, k, min(BLOCK, len(data) - i * BLOCK), s) for i, (k, s) in enumerate(want)]
    assert hashlib.sha256(C.build(cpu)).hexdigest() == hashlib.sha256(got).hexdigest()
