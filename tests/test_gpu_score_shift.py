"""The attention kernels at every range of the score shift, against the CPU oracle (needs a B200).

The kernels compute score = rescale(dot, m, s) in three ways by the shift s of the layer's
attn.score.rescale: a shift of the high word of the 64-bit product for 32 <= s <= 62, a funnel
shift of both words for 21 <= s <= 31, and the general 64-bit rule otherwise. The synthetic models
have s near 40, so this test rewrites each layer's (m, s) to a target shift with about the same
ratio (m >> k, s - k) and checks the weights of prefill groups and decode rows against the
oracle's fast path, for the tensor-core prefill kernel with the decode kernel (HS_ATTN=tc) and
the CUDA-core kernel (HS_ATTN=vec). The output rescale (attn.out.rescale) is checked the same way
at other shifts.
"""

import os

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import synth

pytestmark = pytest.mark.gpu

SEED = 7


@pytest.fixture(scope="module")
def dev():
    d = B.CudaDevice(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def parts():
    fm = synth.float_model(SEED, synth.MINI)
    rg = synth.calibrate(fm, SEED)
    tensors, res = synth.build_tensors(fm, rg)
    eps = max(1, int(round(1e-5 / (res * res) * 2 ** (2 * synth.LN_J))))
    return tensors, eps


def _with_score_shift(parts, target: int, suffix: str = "attn.score.rescale") -> bytes:
    tensors, eps = parts
    out = []
    for name, dt, v, s in tensors:
        if name.endswith(suffix):
            k = s - target
            assert k > 0
            m = np.array([int(v[0]) >> k], np.int32)
            assert m[0] != 0
            out.append((name, dt, m, target))
        else:
            out.append((name, dt, v, s))
    return synth.write_hsm(out, synth.vocabulary(vocab=synth.MINI.vocab), eps, synth.MINI)


def _model(dev, data, attn):
    os.environ["HS_ATTN"] = attn
    try:
        return B.CudaModel(dev, data)
    finally:
        os.environ.pop("HS_ATTN", None)


@pytest.mark.parametrize("attn", ["tc", "vec"])
@pytest.mark.parametrize("shift", [16, 21, 31, 32, 33])
def test_attention_at_each_score_shift_range(dev, parts, attn, shift):
    data = _with_score_shift(parts, shift)
    om = O.Model(data)
    model = _model(dev, data, attn)
    batch = B.CudaBatch(model, 3, 1024)
    fast = O.FastBatch(om, 3, 0)
    rng = np.random.default_rng(shift)
    # A prefill call (groups with ragged ends), then one of decode rows and a short run.
    for spec in ([(0, 200), (1, 130), (2, 33)], [(0, 1), (1, 1), (2, 20), (0, 1)]):
        seq = []
        for s, n in spec:
            seq += [(s, int(t)) for t in rng.integers(0, om.vocab - 1, n)]
        sl = [s for s, _ in seq]
        tk = [t for _, t in seq]
        got = batch.run_weights(sl, tk)
        want = fast.run_weights(sl, tk)
        bad = np.nonzero(~np.all(got == want, axis=1))[0]
        assert bad.size == 0, (attn, shift, bad[:10], len(seq))
    batch.close()
    model.close()


@pytest.mark.parametrize("shift", [31, 32, 47])
def test_attention_at_each_output_shift_range(dev, parts, shift):
    """The output rescale of the attention kernels (a double estimate with an exact 128-bit
    fallback near ties) at output shifts other than the model's own 60."""
    data = _with_score_shift(parts, shift, "attn.out.rescale")
    om = O.Model(data)
    model = _model(dev, data, "tc")
    batch = B.CudaBatch(model, 3, 1024)
    fast = O.FastBatch(om, 3, 0)
    rng = np.random.default_rng(100 + shift)
    for spec in ([(0, 200), (1, 130), (2, 33)], [(0, 1), (1, 1), (2, 20), (0, 1)]):
        seq = []
        for s, n in spec:
            seq += [(s, int(t)) for t in rng.integers(0, om.vocab - 1, n)]
        sl = [s for s, _ in seq]
        tk = [t for _, t in seq]
        got = batch.run_weights(sl, tk)
        want = fast.run_weights(sl, tk)
        bad = np.nonzero(~np.all(got == want, axis=1))[0]
        assert bad.size == 0, (shift, bad[:10], len(seq))
    batch.close()
    model.close()
