"""hs_op_linear_act_noalloc, the linear op staged in the library's static device array, against
the allocating entry point hs_op_linear_act (needs a B200).

The results are integers, so the tolerance is zero: every byte (and every int32 accumulator) must
be equal. Each path is called twice in a row with a large shape and then a smaller one, so stale
operands or padding left in the shared array by the first call would show in the second. The
file is named to be collected last; it passes alone in a fresh process as well.
"""

import numpy as np
import pytest

from taco_b200 import backend as B

pytestmark = pytest.mark.gpu

# (M, N, K): the second shape is smaller in every dimension and ragged against the 128/256 tiles.
SHAPES = [(300, 1024, 768), (77, 256, 200)]


@pytest.fixture(scope="module")
def dev():
    d = B.CudaDevice(0)
    yield d
    d.close()


def _case(rng, M, N, K):
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    W = rng.integers(-128, 128, (N, K), dtype=np.int8)
    b = rng.integers(-(1 << 31), 1 << 31, N, dtype=np.int64).astype(np.int32)
    m = rng.integers(1 << 30, 1 << 31, N, dtype=np.int64).astype(np.int32)
    m[::3] *= -1
    return A, W, b, m


@pytest.mark.parametrize("path", ["tc", "simple"])
def test_noalloc_linear_equals_allocating_entry_point(dev, path):
    rng = np.random.default_rng(2024)
    cases = [_case(rng, *s) for s in SHAPES]
    shift = 38
    got = [dev.linear_act_noalloc(A, W, b, m, shift, path) for A, W, b, m in cases]
    for (A, W, b, m), g in zip(cases, got):
        want = dev.linear_act(A, W, b, m, shift, path)
        assert g.shape == want.shape
        assert np.array_equal(g, want)


@pytest.mark.parametrize("path", ["tc", "simple"])
def test_noalloc_raw_accumulators_equal_allocating_entry_point(dev, path):
    rng = np.random.default_rng(7)
    cases = [_case(rng, *s)[:2] for s in SHAPES]
    got = [dev.linear_act_noalloc(A, W, None, None, 0, path, raw=True) for A, W in cases]
    for (A, W), g in zip(cases, got):
        assert np.array_equal(g, dev.matmul_raw(A, W, path))
        assert np.array_equal(g.astype(np.int64), A.astype(np.int64) @ W.astype(np.int64).T)


def test_noalloc_refuses_shapes_beyond_the_static_array(dev):
    A = np.zeros((8192, 1024), dtype=np.int8)
    W = np.zeros((4096, 1024), dtype=np.int8)
    b = np.zeros(4096, dtype=np.int32)
    with pytest.raises(B.HardShellError) as ei:
        dev.linear_act_noalloc(A, W, b, b, 38, "tc")
    assert ei.value.code == B.HS_UNSUPPORTED
    assert "static scratch" in str(ei.value)
