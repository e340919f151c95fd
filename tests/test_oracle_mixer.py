"""The oracle's weight step of the logs-profile mixer, pinned to the reference's golden vector.

crates/taco-match/tests/golden.rs:44-49 pins the mixer with the SHA-256 of the mixed weights of
every position of a synthetic log (vocab 1000, 4000 tokens, seed 20261018). The weights of a
position come from splitmix64 (tools/logs/vectors.py:46-50 of the reference, restated below); the
prediction and q of each position come from the reference's own Python mirror, recorded by
tests/golden/make_mixer_fixture.py into mixer_v1.bin. The oracle's mix_stats and mix_weights
(the rule 1 and rule 5 weights of taco_match::Mixer::mix) must give the published hash.
"""

import hashlib

import numpy as np

from oracle import oracle as O

from .common import GOLDEN

SEED = 20261018
VOCAB = 1000
TOKENS = 4000
NEWLINE = 198
WEIGHTS_HASH = "31d87e9efc45a331b7019e4c8f6058cea247637a5a29a3b0016981407821d614"  # golden.rs:47
M64 = (1 << 64) - 1
GAMMA, C1, C2 = 0x9E3779B97F4A7C15, 0xBF58476D1CE4E5B9, 0x94D049BB133111EB


class SplitMix64:
    """splitmix64 (the generator of the reference's test vectors)."""

    def __init__(self, seed: int):
        self.state = seed & M64

    def next_u64(self) -> int:
        self.state = (self.state + GAMMA) & M64
        z = self.state
        z = ((z ^ (z >> 30)) * C1) & M64
        z = ((z ^ (z >> 27)) * C2) & M64
        return z ^ (z >> 31)

    def below(self, n: int) -> int:
        return self.next_u64() % n


def splitmix_block(seed: int, count: int) -> np.ndarray:
    """The first `count` outputs of splitmix64(seed), vectorised: output n mixes seed + n * GAMMA."""
    with np.errstate(over="ignore"):
        z = np.uint64(seed & M64) + np.arange(1, count + 1, dtype=np.uint64) * np.uint64(GAMMA)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(C1)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(C2)
    return z ^ (z >> np.uint64(31))


def synthetic_log(seed: int) -> list[int]:
    """The synthetic log of the golden test: 8 templates with variable fields (vectors.py:26-43)."""
    rng = SplitMix64(seed)
    templates = []
    for _ in range(8):
        n = 5 + rng.below(20)
        templates.append([rng.below(VOCAB) for _ in range(n)])
    out: list[int] = []
    while len(out) < TOKENS:
        t = templates[rng.below(8)]
        for tok in t:
            out.append(tok)
            if rng.below(4) == 0:
                for _ in range(1 + rng.below(3)):
                    out.append(rng.below(VOCAB))
        out.append(NEWLINE)
    return out[:TOKENS]


def golden_weights(toks: list[int]) -> np.ndarray:
    """The GPT-2 stand-in weights of every position (vectors.py:46-50): w = x >> (20 + below(44)),
    and w[actual] = 2^40 on a coin flip; 2 * VOCAB + 1 outputs of one generator per position."""
    per = 2 * VOCAB + 1
    z = splitmix_block(SEED ^ 0xA5A5, per * len(toks)).reshape(len(toks), per)
    w = z[:, 0:2 * VOCAB:2] >> (np.uint64(20) + z[:, 1:2 * VOCAB:2] % np.uint64(44))
    flip = z[:, 2 * VOCAB] % np.uint64(2) == 0
    rows = np.nonzero(flip)[0]
    w[rows, np.asarray(toks)[rows]] = np.uint64(1 << 40)
    return w


def test_the_mixed_weights_give_the_published_hash():
    rec = np.fromfile(GOLDEN / "mixer_v1.bin", dtype=np.dtype([("p", "<i4"), ("q", "<u4")]))
    assert rec.size == TOKENS
    toks = synthetic_log(SEED)
    w = golden_weights(toks)
    h = hashlib.sha256()
    mixed = 0
    for i in range(TOKENS):
        p, q = int(rec["p"][i]), int(rec["q"][i])
        if p >= 0:
            total, wp, top = O.mix_stats(w[i], p)
            assert (total, wp, top) == (int(w[i].sum()), int(w[i][p]), int(np.argmax(w[i])))
            out = O.mix_weights(w[i], p, q)
            mixed += 1
        else:
            out = O.mix_weights(w[i], O.MIX_NONE)
        h.update(out.astype("<u8").tobytes())
    assert mixed > 3000
    assert h.hexdigest() == WEIGHTS_HASH


def test_mixed_weight_rules_on_small_rows():
    w = np.array([5, 0, 9, 9, 3], np.uint64)
    assert O.mix_stats(w, 1) == (26, 0, 2)  # the first largest weight
    assert O.mix_stats(np.zeros(4, np.uint64), 3) == (0, 0, 0)
    # R = 26, k = 0: w'[i] = w[i] (2^16 - q) except p, max 1; w'[p] = R q.
    assert O.mix_weights(w, 1, 30000).tolist() == [5 * 35536, 26 * 30000, 9 * 35536, 9 * 35536, 3 * 35536]
    assert O.mix_weights(w, O.MIX_NONE).tolist() == [5, 1, 9, 9, 3]
    assert O.mix_weights(w, O.MIX_PLAIN).tolist() == w.tolist()
    # A large R: k = bitlen(R) + 16 - 62 shifts every product.
    big = np.array([1 << 50, 1 << 40, 3], np.uint64)
    r = (1 << 50) + 3
    k = r.bit_length() + 16 - 62
    want = [((1 << 50) * 100) >> k, (r * 65436) >> k, max(1, (3 * 100) >> k)]
    assert O.mix_weights(big, 1, 65436).tolist() == want
