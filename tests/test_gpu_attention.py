"""The tensor-core prefill attention (head width 64) against the CPU oracle (needs a B200).

The conformance model has 16-wide heads, so these tests use a small synthetic model with GPT-2's
head width (taco_b200/synth.py MINI: 2 layers, d 128, 2 heads, n_ctx 512): prefill groups of 128
rows with ragged ends, groups that start past position 0, the restart rows of a full context with
an overlap, and passes that mix prefill groups with single decode rows. The weights of every row
must equal the oracle's fast path (itself pinned to the reference session), and the CUDA-core
attention (HS_ATTN=vec) must give the same bits.
"""

import os

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mini():
    return synth.gpt2_hsm(7, shape=synth.MINI)


@pytest.fixture(scope="module")
def dev():
    d = B.CudaDevice(0)
    yield d
    d.close()


def _model(dev, data, attn):
    os.environ["HS_ATTN"] = attn
    try:
        return B.CudaModel(dev, data)
    finally:
        os.environ.pop("HS_ATTN", None)


def _batch(model, slots, max_rows, ctas=None):
    """A batch whose persistent attention grid is capped at `ctas` CTAs (HS_ATTN_CTAS), so that
    each CTA runs several tiles of different lengths one after the other."""
    if ctas is not None:
        os.environ["HS_ATTN_CTAS"] = str(ctas)
    try:
        return B.CudaBatch(model, slots, max_rows)
    finally:
        os.environ.pop("HS_ATTN_CTAS", None)


def _calls(rng, vocab):
    """Three calls: long prefill runs, a continuation past position 0 with decode rows mixed in,
    and runs that cross n_ctx = 512 (restarts)."""
    calls = []
    calls.append([(0, 300), (1, 200), (2, 129)])
    calls.append([(1, 1), (0, 140), (2, 1), (1, 1), (2, 40)])
    calls.append([(0, 300), (2, 390), (1, 17)])
    out = []
    for spec in calls:
        seq = []
        for s, n in spec:
            seq += [(s, int(t)) for t in rng.integers(0, vocab - 1, n)]
        out.append(seq)
    return out


@pytest.mark.parametrize("overlap", [0, 20])
@pytest.mark.parametrize("attn,ctas", [("tc", None), ("tc", 1), ("tc", 3), ("vec", None)])
def test_prefill_attention_equals_the_oracle(dev, mini, attn, ctas, overlap):
    om = O.Model(mini)
    model = _model(dev, mini, attn)
    slots = 3
    batch = _batch(model, slots, 1024, ctas)
    batch.set_overlap(overlap)
    fast = O.FastBatch(om, slots, overlap)
    rng = np.random.default_rng(123 + overlap)
    for call, seq in enumerate(_calls(rng, om.vocab)):
        sl = [s for s, _ in seq]
        tk = [t for _, t in seq]
        got = batch.run_weights(sl, tk)
        want = fast.run_weights(sl, tk)
        bad = np.nonzero(~np.all(got == want, axis=1))[0]
        assert bad.size == 0, (attn, overlap, call, bad[:10], len(seq))
        for s in range(slots):
            assert batch.position(s) == fast.position(s)


def test_prefill_coder_answers_tc(dev, mini):
    """The coder answers of a long prefill run (several 128-row groups) with the tensor-core
    attention equal the oracle's."""
    om = O.Model(mini)
    model = _model(dev, mini, "tc")
    batch = B.CudaBatch(model, 1, 512)
    rng = np.random.default_rng(9)
    toks = rng.integers(0, om.vocab - 1, 500)
    kinds = rng.integers(0, 2, toks.size)
    vals = np.where(kinds == 0, rng.integers(0, om.vocab, toks.size),
                    rng.integers(0, 1 << 32, toks.size, dtype=np.uint64))
    got = batch.run_coded(np.zeros(toks.size), toks, kinds, vals, 32)
    fast = O.FastBatch(om, 1, 0)
    want = fast.run_coded(np.zeros(toks.size), toks, kinds, vals, 32)
    assert np.array_equal(got["symbol"].astype(np.uint64), want[:, 0])
    assert np.array_equal(got["start"], want[:, 1])
    assert np.array_equal(got["freq"], want[:, 2])
