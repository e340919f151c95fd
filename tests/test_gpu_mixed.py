"""The mixed coder op of the profile logs on a B200 (crates/hardshell-cuda/src/batch/mixed.rs
run_coded_mixed / run_coded_dual), against the CPU oracle.

For every input the oracle runs the same rows (its fast path's weights), checks the statistics the
device gave the mixer (W, w[p], top: pass 1 of taco_match::Mixer::mix), builds the mixed weights of
the q the mixer returned (the weight step pinned to the reference's golden hash in
test_oracle_mixer.py) and answers the query in FreqTable::from_weights of them. The device answers
must be equal, bit for bit. The cases cover predictions at distance 0 (the top token, a unique max
and a tie), the first and last symbol, q at both ends of 1..=65535 (so that p is, or is not, the
largest symbol), rows without a prediction and plain rows in the same pass, encode and decode
queries (targets at both ends and inside p's interval), prefill and decode passes, a context
restart, a vocabulary of 300, 1000 and 50257 symbols, and freq_bits 32 and 24. Errors: q out of
range, a bad table word, an exception in the mixer; the positions do not move.
"""

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import synth

from .common import tiny_bytes

pytestmark = pytest.mark.gpu

WIDE = synth.Shape(1, 2, 128, 512, 50257, 256)


@pytest.fixture(scope="module")
def dev():
    d = B.CudaDevice(0)
    yield d
    d.close()


def _model_bytes(name):
    if name == "tiny":
        return tiny_bytes()
    if name == "mini":
        return synth.gpt2_hsm(7, shape=synth.MINI)
    return synth.gpt2_hsm(5, shape=WIDE)


class Mixer:
    """A stand-in host mixer: a fixed q per input (from a seeded table), with a log of its calls."""

    def __init__(self, qs):
        self.qs = qs
        self.calls = []

    def __call__(self, i, total, predicted, top):
        self.calls.append((i, total, predicted, top))
        return int(self.qs[i])


def _expected(w, table, q, kind, value, bits):
    if table == O.MIX_PLAIN:
        mixed = w
    elif table == O.MIX_NONE:
        mixed = O.mix_weights(w, O.MIX_NONE)
    else:
        mixed = O.mix_weights(w, table, q)
    return O.answer(mixed, bits, kind, value)


@pytest.mark.parametrize("name,bits", [("tiny", 32), ("mini", 32), ("mini", 24), ("wide", 32)])
def test_mixed_intervals_equal_the_oracle(dev, name, bits):
    data = _model_bytes(name)
    om = O.Model(data)
    V = om.vocab
    rng = np.random.default_rng(len(name) * 100 + bits)
    n_slots, per_slot = 4, 36
    slots = np.repeat(np.arange(n_slots), per_slot)
    rng.shuffle(slots)
    n = slots.size
    tokens = rng.integers(0, V, n)
    # The oracle's weights of every input, in the same order (its slots advance as the device's).
    fast = O.FastBatch(om, n_slots, 0)
    w = fast.run_weights(slots.tolist(), tokens.tolist())
    tables = np.empty(n, np.int64)
    kinds = np.zeros(n, np.int64)
    values = np.zeros(n, np.int64)
    qs = rng.integers(1, 65536, n)
    for i in range(n):
        top = int(np.argmax(w[i]))
        c = i % 12
        tables[i] = {0: top, 1: O.MIX_NONE, 2: O.MIX_PLAIN, 3: 0, 4: V - 1}.get(c, int(rng.integers(0, V)))
        if c in (5, 6):  # a symbol at distance 0 other than the top one, when there is a tie
            ties = np.nonzero(w[i] == w[i][top])[0]
            tables[i] = int(ties[-1])
        if c in (0, 7):
            qs[i] = 65535 if i % 2 else 1  # p the largest symbol, or the others hold nearly all
        if c == 8:
            qs[i] = 1
        kinds[i] = (i // 12) % 2
        if kinds[i] == 0:
            p = tables[i]
            values[i] = {0: p if p < V else 0, 1: top, 2: 0, 3: V - 1}.get(i % 5, int(rng.integers(0, V)))
        else:
            values[i] = {0: 0, 1: (1 << bits) - 1}.get(i % 7, int(rng.integers(0, 1 << bits)))
    # Decode targets inside p's interval for some rows.
    for i in range(0, n, 9):
        if kinds[i] == 1 and tables[i] < V:
            s, start, freq = _expected(w[i], int(tables[i]), int(qs[i]), 0, int(tables[i]), bits)
            values[i] = start + freq // 2
    model = B.CudaModel(dev, data)
    batch = B.CudaBatch(model, n_slots, 64)  # several passes: prefill and decode rows
    mixer = Mixer(qs)
    got = batch.run_coded_mixed(slots, tokens, kinds, values, tables, bits, mixer)
    want_calls = [i for i in range(n) if tables[i] < V]
    assert [c[0] for c in mixer.calls] == want_calls  # input order, token tables only
    for i, total, predicted, top in mixer.calls:
        assert (total, predicted, top) == O.mix_stats(w[i], int(tables[i])), i
    for i in range(n):
        want = _expected(w[i], int(tables[i]), int(qs[i]), int(kinds[i]), int(values[i]), bits)
        g = (int(got["symbol"][i]), int(got["start"][i]), int(got["freq"][i]))
        assert g == want, (i, int(tables[i]), int(kinds[i]), int(values[i]))
        assert got["is_last"][i] == (want[0] == V - 1)
    for s in range(n_slots):
        assert batch.position(s) == fast.position(s)
    batch.close()
    model.close()


def test_dual_gives_the_plain_and_the_mixed_interval(dev):
    data = _model_bytes("mini")
    om = O.Model(data)
    V = om.vocab
    rng = np.random.default_rng(5)
    n_slots = 3
    slots = np.repeat(np.arange(n_slots), 50)
    n = slots.size
    tokens = rng.integers(0, V, n)
    coded = rng.integers(0, V, n)
    preds = np.where(rng.random(n) < 0.3, O.MIX_NONE, rng.integers(0, V, n))
    preds[::7] = coded[::7]  # the prediction is the coded token
    qs = rng.integers(1, 65536, n)
    fast = O.FastBatch(om, n_slots, 0)
    w = fast.run_weights(slots.tolist(), tokens.tolist())
    model = B.CudaModel(dev, data)
    batch = B.CudaBatch(model, n_slots, 128)
    plain, mixed = batch.run_coded_dual(slots, tokens, coded, preds, 32, Mixer(qs))
    for i in range(n):
        assert (int(plain["symbol"][i]), int(plain["start"][i]), int(plain["freq"][i])) == \
            O.answer(w[i], 32, 0, int(coded[i])), i
        want = _expected(w[i], int(preds[i]), int(qs[i]), 0, int(coded[i]), 32)
        assert (int(mixed["symbol"][i]), int(mixed["start"][i]), int(mixed["freq"][i])) == want, i
    batch.close()
    model.close()


def test_mixed_calls_across_a_context_restart(dev):
    data = _model_bytes("mini")
    om = O.Model(data)
    V = om.vocab
    rng = np.random.default_rng(9)
    n = 600  # n_ctx 512: one restart with the overlap
    tokens = rng.integers(0, V, n)
    slots = np.zeros(n, np.int64)
    tables = rng.integers(0, V, n)
    qs = rng.integers(1, 65536, n)
    fast = O.FastBatch(om, 1, 20)
    w = fast.run_weights(slots.tolist(), tokens.tolist())
    model = B.CudaModel(dev, data)
    batch = B.CudaBatch(model, 1, 256)
    batch.set_overlap(20)
    mixer = Mixer(qs)
    got = batch.run_coded_mixed(slots, tokens, np.zeros(n), tokens, tables, 32, mixer)
    assert [c[0] for c in mixer.calls] == list(range(n))
    for i in range(n):
        want = _expected(w[i], int(tables[i]), int(qs[i]), 0, int(tokens[i]), 32)
        assert (int(got["symbol"][i]), int(got["start"][i]), int(got["freq"][i])) == want, i
    assert batch.position(0) == fast.position(0)
    batch.close()
    model.close()


def test_mixed_errors_leave_the_positions(dev):
    model = B.CudaModel(dev, tiny_bytes())
    V = model.info.vocab
    batch = B.CudaBatch(model, 2, 16)
    slots, toks = [0, 1, 0], [5, 6, 7]
    zeros = [0, 0, 0]
    for q in (0, 65536):
        with pytest.raises(B.HardShellError) as e:
            batch.run_coded_mixed(slots, toks, zeros, zeros, [3, 4, 5], 32, lambda *a, q=q: q)
        assert e.value.code == B.HS_UNSUPPORTED
    with pytest.raises(B.HardShellError) as e:
        batch.run_coded_mixed(slots, toks, zeros, zeros, [3, V, 5], 32, lambda *a: 100)
    assert e.value.code == B.HS_UNSUPPORTED
    with pytest.raises(B.HardShellError) as e:
        batch.run_coded_dual(slots, toks, toks, [3, B.MIX_PLAIN, 5], 32, lambda *a: 100)
    assert e.value.code == B.HS_UNSUPPORTED

    def boom(*a):
        raise KeyError("mixer state")

    with pytest.raises(KeyError):
        batch.run_coded_mixed(slots, toks, zeros, zeros, [3, 4, 5], 32, boom)
    assert (batch.position(0), batch.position(1)) == (0, 0)
    # No token table: no mixer call; the plain and none tables still answer.
    calls = []
    got = batch.run_coded_mixed(slots, toks, zeros, zeros, [B.MIX_PLAIN, B.MIX_NONE, B.MIX_NONE], 32,
                                lambda *a: calls.append(a) or 1)
    assert calls == [] and got.size == 3
    assert (batch.position(0), batch.position(1)) == (2, 1)
    batch.close()
    model.close()
