"""Pins the CPU oracle to the reference's own golden data (no GPU).

- the coder golden vector of crates/taco-coder/tests/golden.rs:22-80 (table and stream hashes);
- the conformance model tiny.hsm (its SHA-256 from conformance/README.md);
- every text-profile container of conformance/v2 unfolds to its input, and the coded blocks
  fold again to the same container bytes (crates/taco-cli/tests/conformance.rs checks the same);
- the unit cases of crates/taco-coder/src/freq.rs:280-360.
"""

import hashlib

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import container as C
from tests.common import GOLDEN, splitmix64, tiny_bytes, vectors

TINY_SHA = "eb78b89a4f0f17c7245865aed22f86512a49e0272b7583a831c47e1a401418f8"


def test_manifest_matches_fixture_bytes():
    for line in (GOLDEN / "MANIFEST.tsv").read_text().splitlines():
        name, sha = line.split("\t")
        assert hashlib.sha256((GOLDEN / name).read_bytes()).hexdigest() == sha, name


def test_tiny_model_loads_with_the_published_hash():
    data = tiny_bytes()
    assert hashlib.sha256(data).hexdigest() == TINY_SHA
    m = O.Model(data)
    assert (m.dims["n_layer"], m.dims["d_model"], m.dims["n_head"], m.dims["d_ff"]) == (2, 64, 4, 256)
    assert (m.vocab, m.n_ctx, m.eot) == (300, 64, 299)
    assert m.dims["n_merges"] == 43
    assert m.token_bytes(256 + 8) == b"the"
    assert m.token_bytes(299) == b"<|endoftext|>"


def test_model_loader_refuses_damaged_files():
    data = bytearray(tiny_bytes())
    with pytest.raises(O.OracleError, match="magic"):
        O.Model(b"HSHLMDX\0" + bytes(data[8:]))
    with pytest.raises(O.OracleError):
        O.Model(bytes(data[:-1]))
    bad = bytearray(data)
    bad[-1] ^= 0  # unchanged: still loads
    O.Model(bytes(bad))
    pad = bytearray(data)
    pad[16 + int.from_bytes(data[12:16], "little")] = 1  # a padding byte after the header
    with pytest.raises(O.OracleError, match="padding"):
        O.Model(bytes(pad))


# ---- the coder golden vector (crates/taco-coder/tests/golden.rs) ----

TABLE_A_SHA256 = "6dce098f222c6f262440d5def6ca5bbb7f1cb34c4cef5a26a19835b77c56ff4d"
STREAM_SHA256 = "91676cdc669fca0eb22ed18f5f629882212523261f41d0d5c568b647e78d798f"
STREAM_LEN = 15_689


def _freqs(starts: np.ndarray, bits: int) -> np.ndarray:
    ends = np.append(starts[1:].astype(np.uint64), np.uint64(1 << bits))
    return ends - starts.astype(np.uint64)


def test_coder_golden_stream_has_the_published_hashes():
    s = [0x7AC0C0DE]
    w = []
    for _ in range(1000):
        a = splitmix64(s)
        b = splitmix64(s)
        w.append(a >> (b % 64))
    a_starts = O.from_weights(np.array(w, dtype=np.uint64), 24)
    a_freqs = _freqs(a_starts, 24)
    assert hashlib.sha256(a_freqs.astype("<u8").tobytes()).hexdigest() == TABLE_A_SHA256
    b_starts = np.array([0, 1, (1 << 32) - 1], dtype=np.uint32)
    a_ends = np.cumsum(a_freqs)
    s = [0x5EED]
    ops = []
    for _ in range(20_000):
        x = splitmix64(s)
        r = x % 8
        if r <= 4:
            t = (x >> 8) % (1 << 24)
            ops.append(("A", int(np.searchsorted(a_ends, t, side="right"))))
        elif r == 5:
            ops.append(("B", (x >> 8) % 3))
        else:
            p = (x >> 8) % 4095 + 1
            ops.append(("bit", p, (x >> 40) % 4096 < p))
    enc = O.Encoder()

    def iv(starts, bits, sym):
        n = starts.size
        start = int(starts[sym])
        end = int(starts[sym + 1]) if sym + 1 < n else (1 << bits)
        return start, end - start, sym + 1 == n

    for op in ops:
        if op[0] == "A":
            enc.interval(*iv(a_starts, 24, op[1]), 24)
        elif op[0] == "B":
            enc.interval(*iv(b_starts, 32, op[1]), 32)
        else:
            enc.bit(op[1], op[2])
    data = enc.finish()
    dec = O.Decoder(data)
    for op in ops:
        if op[0] == "A":
            assert dec.table(a_starts, 24) == op[1]
        elif op[0] == "B":
            assert dec.table(b_starts, 32) == op[1]
        else:
            assert dec.bit(op[1]) == op[2]
    assert len(data) == STREAM_LEN
    assert hashlib.sha256(data).hexdigest() == STREAM_SHA256


@pytest.mark.parametrize(
    "weights,bits,freqs",
    [
        ([1, 2, 3, 4], 4, [2, 3, 4, 7]),
        ([3, 3, 1], 3, [4, 3, 1]),
        ([0, 0, 0], 2, [2, 1, 1]),
        ([0, (1 << 64) - 1, 0], 32, [1, (1 << 32) - 2, 1]),
        ([9] * 16, 4, [1] * 16),
        ([5], 32, [1 << 32]),
    ],
)
def test_from_weights_unit_cases(weights, bits, freqs):
    starts = O.from_weights(np.array(weights, dtype=np.uint64), bits)
    assert _freqs(starts, bits).tolist() == freqs


def test_from_weights_refuses_bad_tables():
    with pytest.raises(O.OracleError):
        O.from_weights(np.ones(17, dtype=np.uint64), 4)
    with pytest.raises(O.OracleError):
        O.from_weights(np.zeros(0, dtype=np.uint64), 8)


# ---- the conformance containers ----


def unfold(container: bytes, model: O.Model, decode_coded=None) -> bytes:
    """unfold.rs:125 unfold for the text profile: raw, zstd and coded blocks."""
    c = C.parse(container)
    if c.needs_model:
        assert c.model_hash == hashlib.sha256(model._data).digest()
    out = bytearray()
    for b in c.blocks:
        if b.kind == C.KIND_RAW:
            out += b.stored
        elif b.kind == C.KIND_ZSTD:
            out += C.decode_zstd(b.stored, b.original_len)
        elif b.kind == C.KIND_CODED:
            if decode_coded is None:
                part, _ = O.decode_block(model, b.stored, b.original_len, c.overlap)
            else:
                part = decode_coded(b, c.overlap)
            out += part
        else:
            raise AssertionError("mixed blocks are outside the text profile")
    assert len(out) == c.original_len
    assert hashlib.sha256(bytes(out)).digest() == c.checksum
    return bytes(out)


@pytest.mark.parametrize("vec", vectors(), ids=lambda v: v["name"])
def test_oracle_unfolds_every_text_vector(vec):
    model = O.Model(tiny_bytes())
    data = (GOLDEN / (vec["name"] + ".taco")).read_bytes()
    assert hashlib.sha256(data).hexdigest() == vec["container_sha256"]
    out = unfold(data, model)
    assert out == (GOLDEN / (vec["name"] + ".in")).read_bytes()
    kinds = [C.KIND_NAMES[b.kind] for b in C.parse(data).blocks]
    assert ",".join(kinds) == vec["block_kinds"] or (vec["block_kinds"] == "-" and not kinds)


@pytest.mark.parametrize("name", ["predicted_text_k0", "predicted_text_k32", "all_kinds_text"])
def test_oracle_folds_the_coded_blocks_again(name):
    """The tokens of each coded block, coded again, give the stored payload bit for bit, so the
    container bytes are the published bytes (the encoder side of the pin)."""
    model = O.Model(tiny_bytes())
    data = (GOLDEN / (name + ".taco")).read_bytes()
    c = C.parse(data)
    for b in c.blocks:
        if b.kind != C.KIND_CODED:
            continue
        _, toks = O.decode_block(model, b.stored, b.original_len, c.overlap)
        assert O.encode_block(model, toks, c.overlap) == b.stored
    assert C.build(c) == data


def test_fast_path_equals_the_reference_session():
    """hs_fast (chunks of 32 rows, several slots, restarts with an overlap) gives the weights of
    the reference session for every row (crates/hardshell/tests/fast_paths.rs)."""
    model = O.Model(tiny_bytes())
    rng = np.random.default_rng(7)
    for overlap in (0, 5):
        slots = 3
        fast = O.FastBatch(model, slots, overlap)
        refs = [O.Session(model, overlap) for _ in range(slots)]
        for r in refs:
            r.reset()
        # Three calls: prefill runs of mixed lengths, with restarts past n_ctx = 64.
        for call in range(3):
            sl, tk = [], []
            for s in range(slots):
                n = int(rng.integers(1, 60))
                sl += [s] * n
                tk += rng.integers(0, model.vocab, n).tolist()
            order = rng.permutation(len(sl))
            # Keep each slot's tokens in order while interleaving the slots.
            per = {s: [t for ss, t in zip(sl, tk) if ss == s] for s in range(slots)}
            seq = []
            for i in order:
                s = sl[i]
                seq.append((s, per[s].pop(0)))
            w = fast.run_weights([s for s, _ in seq], [t for _, t in seq])
            for i, (s, t) in enumerate(seq):
                want = refs[s].step(t)
                assert np.array_equal(w[i], want), (overlap, call, i)


def test_fast_path_equals_the_reference_session_on_a_version_2_model():
    """The same on the synthetic version 2 model (16-bit ln_f, fractional betas, a 16-bit GELU
    layer): hs_fast's i8 x i16 products and 16-bit LayerNorm equal the reference session."""
    from taco_b200 import synth

    model = O.Model(synth.gpt2_hsm(7, shape=synth.MINI, wide=True))
    rng = np.random.default_rng(3)
    fast = O.FastBatch(model, 2, 0)
    refs = [O.Session(model, 0) for _ in range(2)]
    seq = [(0, int(t)) for t in rng.integers(0, model.vocab - 1, 40)]
    seq += [(1, int(t)) for t in rng.integers(0, model.vocab - 1, 33)]
    w = fast.run_weights([s for s, _ in seq], [t for _, t in seq])
    for i, (s, t) in enumerate(seq):
        assert np.array_equal(w[i], refs[s].step(t)), i


def test_fast_path_lockstep_lanes_give_the_same_answers():
    """The oracle's lockstep lanes (one decode row for each of up to 8 slots per thread, the CPU
    unfold of crates/taco/src/unfold.rs:215-246) answer as the per-slot path does."""
    om = O.Model(tiny_bytes())
    rng = np.random.default_rng(5)
    slots = 13
    a, b = O.FastBatch(om, slots, 3), O.FastBatch(om, slots, 3)
    pre = rng.integers(0, om.vocab - 1, (slots, 9)).astype(np.uint32)
    sl = np.repeat(np.arange(slots, dtype=np.uint32), 9)
    k0 = np.zeros(sl.size, np.uint32)
    v0 = pre.reshape(-1).astype(np.uint64)
    assert np.array_equal(a.run_coded(sl, pre.reshape(-1), k0, v0, 32, threads=3),
                          b.run_coded(sl, pre.reshape(-1), k0, v0, 32, threads=3))
    one = np.arange(slots, dtype=np.uint32)
    for step in range(4):
        toks = rng.integers(0, om.vocab - 1, slots).astype(np.uint32)
        kinds = np.ones(slots, np.uint32)
        targets = rng.integers(0, 1 << 32, slots, dtype=np.uint64)
        got = a.run_coded(one, toks, kinds, targets, 32, threads=3, lanes=True)
        want = b.run_coded(one, toks, kinds, targets, 32, threads=3)
        assert np.array_equal(got, want), step
