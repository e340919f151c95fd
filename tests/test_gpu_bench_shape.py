"""The bench's own configuration against the oracle: 64 windows of 1,024
tokens of the bench's Zipf text (synth.text_windows, the same seed as bench.py) on the synthetic
GPT-2 124M model, in a batch of 512 slots with passes of 65,536 rows (the bench's default pass:
all 64 windows in one pass), each row coding its next token. The intervals (symbol, start, freq)
of 16 windows spread evenly over the pass, the first and the last among them, equal the CPU
oracle's, field by field; the symbols of every row are the coded tokens. bench.py makes the same
comparison on windows spread over its timed step.
"""

import os

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import synth

pytestmark = pytest.mark.gpu

WINDOWS, WINDOW, CHECKED = 64, 1024, 16


def _rows(windows: np.ndarray, eot: int):
    n_win = windows.shape[0]
    slots = np.repeat(np.arange(n_win, dtype=np.uint32), WINDOW)
    inputs = np.concatenate([np.full((n_win, 1), eot, np.uint32), windows[:, :-1]], axis=1).reshape(-1)
    return slots, inputs, windows.reshape(-1).astype(np.uint64)


def test_bench_shape_intervals_equal_the_oracle():
    model_bytes = synth.gpt2_hsm(124)
    windows = synth.text_windows(WINDOWS, WINDOW, seed=1000)
    eot = synth.VOCAB - 1
    slots, inputs, coded = _rows(windows, eot)
    dev = B.CudaDevice(0)
    model = B.CudaModel(dev, model_bytes)
    batch = B.CudaBatch(model, 512, WINDOWS * WINDOW)
    try:
        got = batch.run_coded(slots, inputs, np.zeros(slots.size, np.uint32), coded, 32)
    finally:
        batch.close()
        model.close()
        dev.close()
    assert np.array_equal(got["symbol"].astype(np.uint64), coded)
    pick = np.linspace(0, WINDOWS - 1, CHECKED).round().astype(np.int64)
    ps, pi, pc = _rows(windows[pick], eot)
    fb = O.FastBatch(O.Model(model_bytes), CHECKED, 0)
    want = fb.run_coded(ps, pi, np.zeros(ps.size, np.uint32), pc, 32, threads=os.cpu_count())
    g = np.stack([got["symbol"], got["start"], got["freq"]], 1).astype(np.uint64)
    g = g.reshape(WINDOWS, WINDOW, 3)[pick].reshape(-1, 3)
    bad = np.flatnonzero(np.any(g != want, axis=1))
    assert bad.size == 0, f"{bad.size} rows differ, first at checked row {bad[:5].tolist()}"
