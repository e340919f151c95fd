// TEST INFRASTRUCTURE ONLY (CPU oracle; see hs_int.hpp).
//
// The fast CPU path of the reference, restated: many independent sessions ("slots") whose rows
// run in chunks of 32 positions (crates/taco/src/fold.rs:24 FOLD_CHUNK, the prefill path of
// crates/hardshell/src/gpt2/session.rs:201 step_many over gpt2/engine.rs:112 forward), with the
// SIMD dot products of crates/hardshell/src/kernels/fast.rs (AVX2 madd_epi16) and the attention
// of gpt2/attention.rs (balanced base-256 digits of p against a transposed values cache).
// The tests prove it equal to the reference session (hs_ref.cpp) row by row; it is the large-case
// checker of the GPU path and the timed CPU baseline.
#pragma once

#include <cstdint>
#include <vector>

#include "hs_model.hpp"

namespace hso {

struct FastBatch {
    const Model* M;
    int slots;
    uint16_t overlap;
    std::vector<int> pos;
    std::vector<uint32_t> hist;  // [slots, n_ctx]
    std::vector<int8_t> kc;      // [slots, L, H, n_ctx, hd]
    std::vector<int8_t> vt;      // [slots, L, H, hd, n_ctx]

    FastBatch(const Model* m, int slots, uint16_t overlap);

    // The inputs (slot[i], token[i]) in order; the rows of one slot run at consecutive positions,
    // with the context restart of gpt2/context.rs. For each input i: with `weights`, its vocab
    // weights at weights[i * vocab]; with `answers`, the coder answer {symbol, start, freq} of
    // query (kind[i], value[i]) at answers[3 * i]. `threads` workers take whole slots; with
    // `lanes` and one row per slot (a decode step), they take groups of up to 8 slots in lockstep
    // (the CPU unfold of crates/taco/src/unfold.rs:215-246). The answers do not depend on it.
    // Returns 0, or 1 (bad slot), 2 (token out of range), 4 (bad query), 5 (bad freq_bits).
    int run(const uint32_t* slot, const uint32_t* token, size_t n, const uint32_t* kind, const uint64_t* value,
            uint32_t bits, uint64_t* answers, uint64_t* weights, int threads, bool lanes);
};

}  // namespace hso
