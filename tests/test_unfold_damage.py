"""Damaged containers through the host unfold, with no GPU (the rule of the reference's
crates/taco/tests/fuzz_unfold.rs damage_case): an unfold of a damaged container gives the
original data exactly, or an error with a short message; never other data, never a crash.

The pool is the conformance containers whose blocks are raw or zstd (their unfold needs no GPU),
and one that names no model. Each case applies one to three seeded damages of these kinds: a bit
flipped, a byte set, the container cut or extended; a header field nudged by one or set to a large
value; a table entry's kind or stored length changed; the length and the block count changed
together so that they agree. Every case runs through the in-memory unfold (an output of at most
1 MiB, as the reference's output limit) and through the pipe unfold. A block that a damage made
coded needs a GPU, which every case refuses (HS_FAIL_OPEN): that is an error like any other here.
"""

import ctypes
import hashlib

import numpy as np
import pytest

from taco_b200 import backend as B
from taco_b200 import container as C

from .common import GOLDEN, tiny_bytes

CASES = 400
OUT_CAP = 1 << 20
ALLOWED = {B.HS_FORMAT, B.HS_CORRUPT, B.HS_MODEL_MISMATCH, B.HS_UNSUPPORTED, B.HS_NO_DEVICE, B.HS_BAD_ARGUMENT}
LARGE = [0, 1, 2**16, 2**31, 2**32 - 1, 2**32, 2**40, 2**63, 2**64 - 1]
# (offset, size) of the header fields of version 2 (crates/taco-format/src/header.rs).
FIELDS = [(4, 2), (6, 2), (40, 8), (80, 4), (84, 4), (88, 1), (89, 1), (90, 2), (92, 1), (93, 1), (94, 2),
          (96, 8)]


def _pool():
    pool = []
    for name in ["empty", "one_byte", "random_raw", "text_k0", "text_k20", "text_kinds"]:
        pool.append(((GOLDEN / (name + ".taco")).read_bytes(), (GOLDEN / (name + ".in")).read_bytes()))
    data = bytes(range(256)) * 3
    c = C.Container(2, bytes(32), len(data), hashlib.sha256(data).digest(), 100)
    c.blocks = [C.Block(i, C.KIND_RAW, len(data[o:o + 100]), data[o:o + 100])
                for i, o in enumerate(range(0, len(data), 100))]
    pool.append((C.build(c), data))
    return pool


def _set(b: bytearray, at: int, size: int, v: int):
    if at + size <= len(b):
        b[at:at + size] = (v % (1 << (8 * size))).to_bytes(size, "little")


def _get(b: bytes, at: int, size: int) -> int:
    return int.from_bytes(b[at:at + size], "little") if at + size <= len(b) else 0


def _damage(rng, b: bytearray):
    kind = int(rng.integers(0, 6))
    if kind <= 1 or len(b) < C.HEADER_LEN:
        if not b:
            b.append(0)
        pos = int(rng.integers(0, len(b)))
        how = int(rng.integers(0, 4))
        if how == 0:
            b[pos] ^= 1 << int(rng.integers(0, 8))
        elif how == 1:
            b[pos] = int(rng.integers(0, 256))
        elif how == 2:
            del b[pos:]
        else:
            b.extend(rng.integers(0, 256, int(rng.integers(1, 9)), dtype=np.uint8).tobytes())
    elif kind == 2:
        at, size = FIELDS[int(rng.integers(0, len(FIELDS)))]
        old = _get(b, at, size)
        v = [old + 1, old - 1, LARGE[int(rng.integers(0, len(LARGE)))]][int(rng.integers(0, 3))]
        _set(b, at, size, v)
    elif kind == 3:
        count = _get(b, 84, 4)
        if count:
            e = C.HEADER_LEN + 5 * int(rng.integers(0, min(count, 1 << 16)))
            if int(rng.integers(0, 2)):
                _set(b, e, 1, int(rng.integers(0, 5)))
            else:
                old = _get(b, e + 1, 4)
                _set(b, e + 1, 4, [old + 1, old - 1, LARGE[int(rng.integers(0, len(LARGE)))]][int(rng.integers(0, 3))])
    else:
        bs = _get(b, 80, 4) or 1
        n = LARGE[int(rng.integers(0, len(LARGE)))]
        _set(b, 40, 8, n)
        _set(b, 84, 4, n // bs + (n % bs != 0))


@pytest.fixture(scope="module")
def tok():
    t = B.Tokenizer(tiny_bytes())
    yield t
    t.close()


def test_damaged_containers_give_the_data_or_an_error(tok, monkeypatch):
    monkeypatch.setenv("HS_FAIL_OPEN", "0")
    pool = _pool()
    model = tiny_bytes()
    ords = np.zeros(1, np.int32)
    out = np.zeros(OUT_CAP, np.uint8)
    n = ctypes.c_size_t()
    tally = {}
    for seed in range(CASES):
        rng = np.random.default_rng(seed)
        container, data = pool[int(rng.integers(0, len(pool)))]
        b = bytearray(container)
        for _ in range(int(rng.integers(1, 4))):
            _damage(rng, b)
        blob = bytes(b)
        # In memory, with an output of at most 1 MiB.
        rc = B.lib().hs_unfold_multi(ords.ctypes.data, 1, model, len(model), 4, 64, tok.h, blob, len(blob),
                                     out.ctypes.data, out.size, ctypes.byref(n))
        if rc == 0:
            assert out[:n.value].tobytes() == data, f"seed {seed}: other data"
        else:
            assert rc in ALLOWED, f"seed {seed}: status {rc}"
            msg = ctypes.create_string_buffer(1024)
            B.lib().hs_last_error(msg, len(msg))
            assert 0 < len(msg.value) <= 400, f"seed {seed}: message {msg.value!r}"
        tally[rc] = tally.get(rc, 0) + 1
        # Through a pipe, with the same output limit.
        got = bytearray()

        def write(chunk):
            if len(got) + len(chunk) > OUT_CAP:
                raise OSError("over the output limit")
            got.extend(chunk)

        pos = [0]

        def read(k):
            piece = blob[pos[0]:pos[0] + min(k, 777)]
            pos[0] += len(piece)
            return piece

        try:
            B.unfold_pipe_multi([0], model, tok, read, write)
            assert bytes(got) == data, f"seed {seed}: the pipe gave other data"
        except B.HardShellError as e:
            assert e.code in ALLOWED | {B.HS_IO}, f"seed {seed}: pipe status {e.code}"
    # The damages reach the data (some cases are refused, some still unfold to the original).
    assert tally.get(0, 0) > 0 and sum(v for k, v in tally.items() if k) > CASES // 2, tally
