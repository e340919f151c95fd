"""Record the mixer decisions that pin the oracle's mixed weights to the reference's golden vector.

Run once in a container that has the reference checkout (its path is the first argument):

    python tests/golden/make_mixer_fixture.py <reference checkout>

The reference pins its mixer with the SHA-256 of all mixed weights of a synthetic log
(crates/taco-match/tests/golden.rs:44-49, seed 20261018, 4000 tokens, vocab 1000), and its Python
mirror (tools/logs/vectors.py) gives the same hash. The mixed weights of a row depend on its
GPT-2 weights (splitmix64, easy to regenerate), the match model's prediction, and the mixer's q
(the adaptive state machine of rules 2 to 4 and 6, outside the GPU path). This script runs the
reference's Python mirror, checks that it still gives the published hashes, and writes, for each
of the 4000 positions, the prediction (-1 for none) and q as little-endian int32 / uint32 pairs
into mixer_v1.bin. tests/test_oracle_mixer.py regenerates the weights, applies the oracle's weight
step with these (prediction, q) pairs, and must reach the published hash.
"""

import struct
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SEED = 20261018
# crates/taco-match/tests/golden.rs:46-47, v1_parameters_match_the_python_mirror.
PRED_HASH = "a7ccc360407bc350f5444defc5dcb8b173ec6e7ee8c17b02998d70c20c73b23d"
WEIGHTS_HASH = "31d87e9efc45a331b7019e4c8f6058cea247637a5a29a3b0016981407821d614"


def main() -> int:
    sys.path.insert(0, str(Path(sys.argv[1]) / "tools"))
    from convert.rng import SplitMix64
    from logs import matchmodel as mm
    from logs import mixer as mx
    from logs import vectors as vec

    v1 = mm.MatchParams((32, 16, 8, 4, 2, 1), 20, 64, 65535)
    assert vec.run(SEED, v1, mx.MixerParams()) == (PRED_HASH, WEIGHTS_HASH), "the mirror moved"
    # The loop of vectors.run, recording what the weight step gets.
    toks = vec.tokens(SEED)
    pred, plen = mm.predict_block_ref(toks, v1)
    rng = SplitMix64(SEED ^ 0xA5A5)
    m = mx.Mixer(mx.MixerParams())
    out = bytearray()
    for i, t in enumerate(toks):
        w = vec.weights(rng, t)
        q = 0
        if pred[i] >= 0:
            top = max(range(vec.VOCAB), key=lambda j: (w[j], -j))
            q = m.prob(w[pred[i]], sum(w), plen[i], top == pred[i])
            m.update(pred[i] == t)
        out += struct.pack("<iI", pred[i], q)
    (HERE / "mixer_v1.bin").write_bytes(bytes(out))
    print(f"wrote {len(toks)} positions to mixer_v1.bin")
    return 0


if __name__ == "__main__":
    sys.exit(main())
