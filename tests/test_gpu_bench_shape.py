"""The bench's own configuration against the oracle: 16 windows of 1,024
tokens of the bench's Zipf text (synth.text_windows, the same seed as bench.py) on the synthetic
GPT-2 124M model, in a batch of 512 slots with passes of 16,384 rows (one full pass), each row
coding its next token. The intervals (symbol, start, freq) of every row equal the CPU oracle's,
field by field. bench.py makes the same comparison on the first windows of its timed run.
"""

import os

import numpy as np
import pytest

from oracle import oracle as O
from taco_b200 import backend as B
from taco_b200 import synth

pytestmark = pytest.mark.gpu

WINDOWS, WINDOW = 16, 1024


def test_bench_shape_intervals_equal_the_oracle():
    model_bytes = synth.gpt2_hsm(124)
    windows = synth.text_windows(WINDOWS, WINDOW, seed=1000)
    eot = synth.VOCAB - 1
    slots = np.repeat(np.arange(WINDOWS, dtype=np.uint32), WINDOW)
    inputs = np.concatenate([np.full((WINDOWS, 1), eot, np.uint32), windows[:, :-1]], axis=1).reshape(-1)
    coded = windows.reshape(-1).astype(np.uint64)
    dev = B.CudaDevice(0)
    model = B.CudaModel(dev, model_bytes)
    batch = B.CudaBatch(model, 512, 16384)
    try:
        got = batch.run_coded(slots, inputs, np.zeros(slots.size, np.uint32), coded, 32)
    finally:
        batch.close()
        model.close()
        dev.close()
    om = O.Model(model_bytes)
    fb = O.FastBatch(om, WINDOWS, 0)
    want = fb.run_coded(slots, inputs, np.zeros(slots.size, np.uint32), coded, 32, threads=os.cpu_count())
    g = np.stack([got["symbol"], got["start"], got["freq"]], 1).astype(np.uint64)
    bad = np.flatnonzero(np.any(g != want, axis=1))
    assert bad.size == 0, f"{bad.size} rows differ, first at row {bad[:5].tolist()}"
    assert np.array_equal(got["symbol"].astype(np.uint64), coded)
