"""Version 2 ("wide") models on the GPU against the CPU oracle (needs a B200).

A version 2 .hsm (crates/hardshell/src/hsm/reader.rs check_version) may have a 16-bit final
LayerNorm (ln_f_bits = 16), LayerNorm betas with fractional bits (ln_beta_frac) and 16-bit GELU
tables. The backend carries each i16 activation as two i8 planes, v = 256 hi + lo + 128, and
recombines the two tcgen05 accumulators exactly (crates/hardshell/src/kernels.rs:91
matvec_i8_i16). The synthetic model (taco_b200/synth.py, wide=True) has all three: ln_f_bits
16, ln_beta_frac 4 with non-zero betas, and 16-bit GELU in layer 0 (8-bit in layer 1). Every
weight and every coder answer must equal the oracle's.
"""

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def wide():
    return synth.gpt2_hsm(7, shape=synth.MINI, wide=True)


@pytest.fixture(scope="module")
def dev():
    d = B.CudaDevice(0)
    yield d
    d.close()


def test_wide_model_loads_as_version_2(dev, wide):
    model = B.CudaModel(dev, wide)
    assert model.info.version == 2


@pytest.mark.parametrize("overlap", [0, 20])
def test_wide_weights_equal_the_oracle(dev, wide, overlap):
    om = O.Model(wide)
    model = B.CudaModel(dev, wide)
    slots = 3
    batch = B.CudaBatch(model, slots, 1024)
    batch.set_overlap(overlap)
    fast = O.FastBatch(om, slots, overlap)
    rng = np.random.default_rng(5 + overlap)
    calls = [[(0, 300), (1, 130), (2, 1)], [(1, 1), (0, 140), (2, 3), (1, 1)], [(0, 200), (2, 380), (1, 17)]]
    for call, spec in enumerate(calls):
        seq = []
        for s, n in spec:
            seq += [(s, int(t)) for t in rng.integers(0, om.vocab - 1, n)]
        sl = [s for s, _ in seq]
        tk = [t for _, t in seq]
        got = batch.run_weights(sl, tk)
        want = fast.run_weights(sl, tk)
        bad = np.nonzero(~np.all(got == want, axis=1))[0]
        assert bad.size == 0, (overlap, call, bad[:10], len(seq))


def test_wide_coder_answers_equal_the_oracle(dev, wide):
    om = O.Model(wide)
    model = B.CudaModel(dev, wide)
    batch = B.CudaBatch(model, 2, 512)
    rng = np.random.default_rng(11)
    n = 400
    slots = np.repeat(np.arange(2), n // 2).astype(np.uint32)
    toks = rng.integers(0, om.vocab - 1, n)
    kinds = rng.integers(0, 2, n)
    vals = np.where(kinds == 0, rng.integers(0, om.vocab, n), rng.integers(0, 1 << 32, n, dtype=np.uint64))
    got = batch.run_coded(slots, toks, kinds, vals, 32)
    fast = O.FastBatch(om, 2, 0)
    want = fast.run_coded(slots, toks, kinds, vals, 32)
    assert np.array_equal(got["symbol"].astype(np.uint64), want[:, 0])
    assert np.array_equal(got["start"], want[:, 1])
    assert np.array_equal(got["freq"], want[:, 2])
