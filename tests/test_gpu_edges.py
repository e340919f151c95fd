"""Edge cases of the batch calls against the CPU oracle (needs a B200).

- An empty call returns nothing and moves no position (crates/hardshell-cuda/src/batch.rs run:
  no input, no pass).
- A call with more rows than the batch's max_rows runs as several passes and gives the same
  weights as one oracle call.
- Batched decode: 64 streams of different lengths, then decode steps of one row per stream. Every
  32-row group of those passes mixes slots, so the values cache is written through the staging
  rows and the scatter kernel, and attention takes the decode kernel.
- Decode queries at the ends of the target range (0 and 2^bits - 1) and encode queries of the
  first and last symbol of the vocabulary.
"""

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import synth

from .common import tiny_bytes

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    d = B.CudaDevice(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def mini():
    return synth.gpt2_hsm(7, shape=synth.MINI)


def _same(got, want):
    bad = np.nonzero(~np.all(got == want, axis=1))[0]
    assert bad.size == 0, (bad[:10], len(got))


def test_empty_calls_return_nothing_and_move_nothing(dev):
    model = B.CudaModel(dev, tiny_bytes())
    batch = B.CudaBatch(model, 2, 16)
    batch.run_weights([0, 0, 1], [5, 6, 7])
    w = batch.run_weights([], [])
    assert w.shape == (0, model.vocab_size())
    iv = batch.run_coded([], [], [], [], 32)
    assert iv.shape == (0,)
    assert (batch.position(0), batch.position(1)) == (2, 1)
    batch.close()
    model.close()


def test_a_call_longer_than_max_rows_runs_as_several_passes(dev):
    data = tiny_bytes()
    model = B.CudaModel(dev, data)
    om = O.Model(data)
    batch = B.CudaBatch(model, 3, 16)
    fast = O.FastBatch(om, 3, 0)
    rng = np.random.default_rng(5)
    for n in (40, 17, 33):
        sl = rng.integers(0, 3, n).tolist()
        tk = rng.integers(0, om.vocab - 1, n).tolist()
        _same(batch.run_weights(sl, tk), fast.run_weights(sl, tk))
    assert [batch.position(s) for s in range(3)] == [fast.position(s) for s in range(3)]
    batch.close()
    model.close()


def test_batched_decode_of_many_streams_equals_the_oracle(dev, mini):
    om = O.Model(mini)
    model = B.CudaModel(dev, mini)
    streams = 64
    batch = B.CudaBatch(model, streams, 4096)
    fast = O.FastBatch(om, streams, 0)
    rng = np.random.default_rng(11)
    lens = rng.integers(1, 200, streams)
    sl = np.repeat(np.arange(streams), lens).tolist()
    tk = rng.integers(0, om.vocab - 1, len(sl)).tolist()
    _same(batch.run_weights(sl, tk), fast.run_weights(sl, tk))
    order = np.arange(streams)
    for step in range(4):
        rng.shuffle(order)  # the rows of a pass need not be in slot order
        sl = order.tolist()
        tk = rng.integers(0, om.vocab - 1, streams).tolist()
        _same(batch.run_weights(sl, tk), fast.run_weights(sl, tk))
    assert [batch.position(s) for s in range(streams)] == [fast.position(s) for s in range(streams)]
    batch.close()
    model.close()


@pytest.mark.parametrize("bits", [32, 24])
def test_coder_queries_at_the_ends_of_their_ranges(dev, mini, bits):
    om = O.Model(mini)
    model = B.CudaModel(dev, mini)
    batch = B.CudaBatch(model, 4, 64)
    fast = O.FastBatch(om, 4, 0)
    top = (1 << bits) - 1
    sl = [0, 1, 2, 3, 0, 1, 2, 3]
    tk = [1, 2, 3, 4, 5, 6, 7, 8]
    kinds = [1, 1, 0, 0, 1, 0, 1, 0]
    values = [0, top, 0, om.vocab - 1, top, om.vocab - 1, 0, 0]
    got = batch.run_coded(sl, tk, kinds, values, bits)
    want = fast.run_coded(sl, tk, kinds, values, bits)  # (symbol, start, freq) per row
    for i, f in enumerate(("symbol", "start", "freq")):
        assert np.array_equal(got[f].astype(np.uint64), want[:, i]), f
    assert np.array_equal(got["is_last"] != 0, want[:, 0] == om.vocab - 1)
    batch.close()
    model.close()


def test_one_pass_of_more_than_65535_rows(dev):
    """A pass of 70,400 rows (1,100 slots x 64 positions of the tiny model, max_rows 70,400): the
    kernels index rows in the first grid dimension, so a pass may hold up to max_rows (2^20)
    rows. Every coder answer equals the oracle's."""
    slots, n = 1100, 64
    rng = np.random.default_rng(65536)
    toks = rng.integers(0, 299, (slots, n)).astype(np.uint32)
    sl = np.repeat(np.arange(slots, dtype=np.uint32), n)
    inputs = np.concatenate([np.full((slots, 1), 299, np.uint32), toks[:, :-1]], axis=1).reshape(-1)
    coded = toks.reshape(-1).astype(np.uint64)
    model = B.CudaModel(dev, tiny_bytes())
    batch = B.CudaBatch(model, slots, slots * n)
    try:
        got = batch.run_coded(sl, inputs, np.zeros(sl.size, np.uint32), coded, 32)
    finally:
        batch.close()
        model.close()
    fb = O.FastBatch(O.Model(tiny_bytes()), slots, 0)
    want = fb.run_coded(sl, inputs, np.zeros(sl.size, np.uint32), coded, 32)
    _same(np.stack([got["symbol"], got["start"], got["freq"]], 1).astype(np.uint64), want)
