"""Truncation of a slot, the engine side of speculative decoding (crates/hardshell-cuda/src/batch/
stream.rs; rules of crates/hardshell/src/gpt2/stream.rs), on a B200.

The defining property: after truncate(slot, len) the slot gives the weights of a slot that ran
only its first `len` inputs, bit for bit. It is checked against a fresh slot that ran those
inputs and against the CPU oracle, both inside the current context and back across a context
restart (the old context taken back and its overwritten rows run again). Errors leave the slot
unchanged. stream_len and room follow the reference's counts.
"""

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import synth

pytestmark = pytest.mark.gpu

OVERLAP = 20


@pytest.fixture(scope="module")
def dev():
    d = B.CudaDevice(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def mini():
    return synth.gpt2_hsm(7, shape=synth.MINI)


def _run(batch, slot, toks, chunk=256):
    """Runs the tokens through one slot in calls of at most `chunk` inputs; the weights of all."""
    out = []
    for i in range(0, len(toks), chunk):
        part = [int(t) for t in toks[i:i + chunk]]
        out.append(batch.run_weights([slot] * len(part), part))
    return np.concatenate(out) if out else np.zeros((0, 0), np.uint64)


@pytest.mark.parametrize("total,keep", [(55, 40), (60, 60), (600, 500), (600, 560), (700, 470)])
def test_truncated_slot_equals_a_slot_that_ran_only_the_kept_inputs(dev, mini, total, keep):
    om = O.Model(mini)
    model = B.CudaModel(dev, mini)
    batch = B.CudaBatch(model, 2, 1024)
    batch.set_overlap(OVERLAP)
    rng = np.random.default_rng(total * 7 + keep)
    toks = rng.integers(0, om.vocab - 1, total)
    more = rng.integers(0, om.vocab - 1, 15)
    _run(batch, 0, toks)
    assert batch.stream_len(0) == total
    batch.truncate(0, keep)
    assert batch.stream_len(0) == keep
    got = _run(batch, 0, more)
    _run(batch, 1, toks[:keep])
    want = _run(batch, 1, more)
    assert batch.position(0) == batch.position(1)
    assert np.array_equal(got, want)
    fast = O.FastBatch(om, 1, OVERLAP)
    _run(fast, 0, toks[:keep])
    assert np.array_equal(got, _run(fast, 0, more))
    batch.close()
    model.close()


def test_truncation_errors_leave_the_slot_unchanged(dev, mini):
    om = O.Model(mini)
    model = B.CudaModel(dev, mini)
    batch = B.CudaBatch(model, 2, 1024)
    batch.set_overlap(OVERLAP)
    rng = np.random.default_rng(3)
    toks = rng.integers(0, om.vocab - 1, 1100)  # two context restarts
    _run(batch, 0, toks)
    pos = batch.position(0)
    with pytest.raises(B.HardShellError) as e:
        batch.truncate(0, 1101)  # longer than the stream
    assert e.value.code == B.HS_MODEL
    with pytest.raises(B.HardShellError) as e:
        batch.truncate(0, 100)  # before the restart before the last one
    assert e.value.code == B.HS_MODEL
    with pytest.raises(B.HardShellError) as e:
        batch.truncate(5, 1)
    assert e.value.code == B.HS_BAD_SLOT
    assert (batch.position(0), batch.stream_len(0)) == (pos, 1100)
    batch.close()
    model.close()


def test_room_and_stream_length(dev, mini):
    model = B.CudaModel(dev, mini)
    n_ctx = model.n_ctx()
    batch = B.CudaBatch(model, 1, 1024)
    batch.set_overlap(OVERLAP)
    assert (batch.room(0), batch.stream_len(0)) == (n_ctx, 0)
    _run(batch, 0, np.arange(50) % 100)
    assert (batch.room(0), batch.stream_len(0)) == (n_ctx - 50, 50)
    _run(batch, 0, np.arange(n_ctx - 50) % 100)
    assert batch.position(0) == n_ctx
    assert batch.room(0) == n_ctx - OVERLAP - 1  # the next input restarts first
    batch.reset(0)
    assert (batch.room(0), batch.stream_len(0)) == (n_ctx, 0)
    toks, status = batch.decode_blocks([0], [bytes(range(64))], [30], 32)
    assert batch.stream_len(0) == 30 and batch.position(0) == 30
    batch.close()
    model.close()
