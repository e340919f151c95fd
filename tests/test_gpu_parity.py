"""Parity of the CUDA path with the CPU oracle (needs a B200).

- the int8 GEMM (tensor cores and CUDA cores) against exact numpy sums and the requant rule;
- the full forward pass on the conformance model tiny.hsm: weights and coder answers of every
  row against the oracle, with prefill, several slots and context restarts with an overlap;
- unfold and fold of the conformance containers through the C ABI: the same bytes as the
  reference (crates/taco-cli/tests/conformance.rs; crates/hardshell-cuda/tests/gpt2.rs);
- the errors of the boundary (crates/hardshell-cuda/src/error.rs) and the transactional rule.
"""

import hashlib
import os

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import container as C
from tests.common import GOLDEN, tiny_bytes, vectors

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    d = B.CudaDevice(0)
    yield d
    d.close()


def requant_act(acc: np.ndarray, b: np.ndarray, m: np.ndarray, s: int) -> np.ndarray:
    """ops.rs:434 LinearOut::Act: clamp(floor((acc + b) * m + 2^(s-1)) / 2^s), -127, 127)."""
    p = (acc.astype(np.int64) + b.astype(np.int64)) * m.astype(np.int64)
    if s == 0:
        y = p
    elif s >= 64:
        y = np.zeros_like(p)
    else:
        y = (p >> s) + ((p >> (s - 1)) & 1)
    return np.clip(y, -127, 127).astype(np.int8)


@pytest.mark.parametrize("path", ["tc", "simple"])
@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (5, 192, 64), (128, 768, 768), (300, 2304, 768),
                                   (257, 768, 3072), (130, 512, 300)])
def test_gemm_exact_int32(dev, path, M, N, K):
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    W = rng.integers(-128, 128, (N, K), dtype=np.int8)
    if N % 16 and path == "tc":
        pytest.skip("the op-level tensor-core entry needs N % 16 == 0")
    got = dev.matmul_raw(A, W, path)
    want = A.astype(np.int64) @ W.astype(np.int64).T
    assert np.array_equal(got.astype(np.int64), want)


@pytest.mark.parametrize("path", ["tc", "simple"])
def test_gemm_extremes(dev, path):
    K = 2048
    A = np.full((130, K), -128, dtype=np.int8)
    W = np.full((256, K), -128, dtype=np.int8)
    W[1::2] = 127
    got = dev.matmul_raw(A, W, path)
    want = A.astype(np.int64) @ W.astype(np.int64).T
    assert np.array_equal(got.astype(np.int64), want)


@pytest.mark.parametrize("path", ["tc", "simple"])
@pytest.mark.parametrize("shift", [0, 22, 31, 38, 63, 70])
def test_linear_requant(dev, path, shift):
    rng = np.random.default_rng(shift)
    M, N, K = 200, 768, 768
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    W = rng.integers(-128, 128, (N, K), dtype=np.int8)
    b = rng.integers(-(1 << 31), 1 << 31, N, dtype=np.int64).astype(np.int32)
    m = rng.integers(1 << 30, 1 << 31, N, dtype=np.int64).astype(np.int32)
    m[::3] *= -1
    got = dev.linear_act(A, W, b, m, shift, path)
    want = requant_act(A.astype(np.int64) @ W.astype(np.int64).T, b, m, shift)
    assert np.array_equal(got, want)


def _model(dev, path):
    os.environ["HS_GEMM"] = path
    try:
        return B.CudaModel(dev, tiny_bytes())
    finally:
        os.environ.pop("HS_GEMM", None)


@pytest.mark.parametrize("path", ["tc", "simple"])
@pytest.mark.parametrize("overlap", [0, 7])
def test_forward_weights_equal_the_oracle(dev, path, overlap):
    """Every row's weights equal the reference session's, bit for bit: prefill runs of several
    slots in one call, passes split by max_rows, and restarts past n_ctx = 64."""
    om = O.Model(tiny_bytes())
    model = _model(dev, path)
    slots = 3
    batch = B.CudaBatch(model, slots, 40)
    batch.set_overlap(overlap)
    refs = [O.Session(om, overlap) for _ in range(slots)]
    rng = np.random.default_rng(11 + overlap)
    for call in range(4):
        seq = []
        for s in range(slots):
            n = int(rng.integers(1, 50))
            seq += [(s, int(t)) for t in rng.integers(0, om.vocab, n)]
        # Interleave the slots, keeping each slot's tokens in order.
        order = sorted(range(len(seq)), key=lambda i: (rng.random(), 0))
        per = {s: [t for ss, t in seq if ss == s] for s in range(slots)}
        mixed = []
        for i in order:
            s = seq[i][0]
            mixed.append((s, per[s].pop(0)))
        w = batch.run_weights([s for s, _ in mixed], [t for _, t in mixed])
        for i, (s, t) in enumerate(mixed):
            want = refs[s].step(t)
            assert np.array_equal(w[i], want), (path, overlap, call, i)
        for s in range(slots):
            assert batch.position(s) == refs[s].position


@pytest.mark.parametrize("path", ["tc", "simple"])
def test_coder_answers_equal_the_oracle(dev, path):
    """The coder op gives the interval of FreqTable::from_weights for Encode and Decode queries,
    with freq_bits 32 and a smaller total."""
    om = O.Model(tiny_bytes())
    model = _model(dev, path)
    batch = B.CudaBatch(model, 2, 64)
    ref = O.Session(om, 0)
    rng = np.random.default_rng(5)
    toks = rng.integers(0, om.vocab, 60)
    for bits in (32, 20, 9):
        batch.reset(0)
        ref.reset()
        kinds = rng.integers(0, 2, toks.size)
        vals = np.where(kinds == 0, rng.integers(0, om.vocab, toks.size),
                        rng.integers(0, 1 << bits, toks.size, dtype=np.uint64))
        got = batch.run_coded(np.zeros(toks.size), toks, kinds, vals, bits)
        for i, t in enumerate(toks):
            w = ref.step(int(t))
            want = O.answer(w, bits, int(kinds[i]), int(vals[i]))
            assert (int(got[i]["symbol"]), int(got[i]["start"]), int(got[i]["freq"])) == want, (bits, i)
            assert bool(got[i]["is_last"]) == (want[0] == om.vocab - 1)


def _gpu_decode_block(batch, model_vocab, payload: bytes, original_len: int, om: O.Model, eot: int) -> bytes:
    """codec.rs BlockDecoder with the GPU coder op: one run_coded call per token (Decode)."""
    varint_end = next(i for i, byte in enumerate(payload) if byte < 0x80) + 1
    count = 0
    for i, byte in enumerate(payload[:varint_end]):
        count |= (byte & 0x7F) << (7 * i)
    dec = O.Decoder(payload[varint_end:])
    batch.reset(0)
    out = bytearray()
    token = eot
    for _ in range(count):
        target = dec.target(32)
        a = batch.run_coded([0], [token], [B.DECODE], [target], 32)[0]
        sym = int(a["symbol"])
        assert dec.interval(int(a["start"]), int(a["freq"]), bool(a["is_last"]), 32)
        out += om.token_bytes(sym)
        token = sym
    assert len(out) == original_len
    return bytes(out)


@pytest.mark.parametrize("name", ["predicted_text_k0", "predicted_text_k32", "all_kinds_text"])
def test_gpu_unfolds_the_conformance_containers(dev, name):
    om = O.Model(tiny_bytes())
    model = B.CudaModel(dev, tiny_bytes())
    assert model.hash() == hashlib.sha256(tiny_bytes()).digest()
    data = (GOLDEN / (name + ".taco")).read_bytes()
    c = C.parse(data)
    assert c.model_hash == model.hash()
    batch = B.CudaBatch(model, 1, 8)
    batch.set_overlap(c.overlap)
    out = bytearray()
    for b in c.blocks:
        if b.kind == C.KIND_RAW:
            out += b.stored
        elif b.kind == C.KIND_ZSTD:
            out += C.decode_zstd(b.stored, b.original_len)
        else:
            out += _gpu_decode_block(batch, om.vocab, b.stored, b.original_len, om, om.eot)
    assert bytes(out) == (GOLDEN / (name + ".in")).read_bytes()
    assert hashlib.sha256(bytes(out)).digest() == c.checksum


@pytest.mark.parametrize("name", ["predicted_text_k0", "predicted_text_k32", "all_kinds_text"])
def test_gpu_folds_the_coded_blocks_to_the_published_container(dev, name):
    """All tokens of a block in one prefill call (Encode queries), intervals into the range
    encoder: the payload and the container are the published bytes."""
    om = O.Model(tiny_bytes())
    model = B.CudaModel(dev, tiny_bytes())
    data = (GOLDEN / (name + ".taco")).read_bytes()
    c = C.parse(data)
    batch = B.CudaBatch(model, 1, 512)
    batch.set_overlap(c.overlap)
    for b in c.blocks:
        if b.kind != C.KIND_CODED:
            continue
        _, toks = O.decode_block(om, b.stored, b.original_len, c.overlap)
        batch.reset(0)
        inputs = [om.eot] + toks[:-1]
        ans = batch.run_coded(np.zeros(len(toks)), inputs, np.zeros(len(toks)), toks, 32)
        enc = O.Encoder()
        for a, t in zip(ans, toks):
            assert int(a["symbol"]) == t
            enc.interval(int(a["start"]), int(a["freq"]), bool(a["is_last"]), 32)
        n = len(toks)
        varint = bytearray()
        while True:
            low = n & 0x7F
            n >>= 7
            if n == 0:
                varint.append(low)
                break
            varint.append(low | 0x80)
        assert bytes(varint) + enc.finish() == b.stored
    assert C.build(c) == data


def test_boundary_errors_and_transactions(dev):
    model = B.CudaModel(dev, tiny_bytes())
    batch = B.CudaBatch(model, 2, 16)
    with pytest.raises(B.HardShellError) as e:
        batch.run_weights([2], [1])
    assert e.value.code == B.HS_BAD_SLOT
    batch.run_weights([0, 0, 1], [5, 6, 7])
    assert (batch.position(0), batch.position(1)) == (2, 1)
    with pytest.raises(B.HardShellError) as e:
        batch.run_weights([0, 1], [3, model.vocab_size()])
    assert e.value.code == B.HS_TOKEN_RANGE
    assert (batch.position(0), batch.position(1)) == (2, 1)  # no position changed
    with pytest.raises(B.HardShellError) as e:
        batch.run_coded([0], [3], [0], [model.vocab_size()], 32)
    assert e.value.code == B.HS_UNSUPPORTED
    with pytest.raises(B.HardShellError) as e:
        batch.run_coded([0], [3], [1], [1 << 20], 20)
    assert e.value.code == B.HS_UNSUPPORTED
    with pytest.raises(B.HardShellError) as e:
        batch.run_coded([0], [3], [0], [1], 8)  # 2^8 < vocab 300
    assert e.value.code == B.HS_UNSUPPORTED
    with pytest.raises(B.HardShellError) as e:
        batch.set_overlap(model.n_ctx() - 1)
    assert e.value.code == B.HS_INVALID_OVERLAP
    assert (batch.position(0), batch.position(1)) == (2, 1)
    with pytest.raises(B.HardShellError) as e:
        B.CudaModel(dev, tiny_bytes()[:-1])
    assert e.value.code == B.HS_MODEL
