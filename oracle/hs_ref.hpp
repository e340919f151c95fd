// TEST INFRASTRUCTURE ONLY (CPU oracle; see hs_int.hpp).
//
// The reference forward pass of HardShell (the oracle of the reference itself,
// crates/hardshell/src/gpt2/reference.rs) and the coder of crates/taco-coder.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "hs_model.hpp"

namespace hso {

// layernorm.rs:201 LayerNorm::apply_with. `out16` selects the i16 clamp (apply_i16).
void layernorm_apply(const Model& M, const LayerNormP& ln, const int32_t* x, int8_t* out8, int16_t* out16);

// softmax.rs:78 softmax. Returns false on the reference's error cases.
bool softmax_ref(const int64_t* scores, size_t n, const std::vector<int32_t>& table, uint32_t p, int64_t* out);

// logits.rs:62 logits_to_weights.
void logits_to_weights(const int64_t* logits, size_t n, const std::vector<uint64_t>& table, uint64_t* out);

// gpt2/reference.rs:23 ReferenceSession: one token at a time, with the scalar kernels.
struct RefSession {
    const Model* model;
    uint16_t overlap = 0;
    int pos = 0;
    std::vector<uint32_t> tokens;
    std::vector<int8_t> k_cache, v_cache;  // [n_layer, n_ctx, d]
    std::vector<int32_t> x;
    std::vector<int8_t> a;
    std::vector<int16_t> a16;
    std::vector<int8_t> qkv, att, g;
    std::vector<int16_t> g16;
    std::vector<int64_t> scores, probs, head_acc, logits;
    std::vector<uint64_t> weights;

    RefSession(const Model* m, uint16_t k);
    void reset() { pos = 0; }
    // reference.rs:144 step. Returns 0, or an error code (1 token out of range,
    // 2 invalid overlap).
    int step(uint32_t token);
    int start_block() {
        reset();
        return step(model->eot);
    }

   private:
    void forward(uint32_t tok, bool logits);
    void embed(uint32_t tok, int t);
    void attention(int layer, int t);
    void mlp(int layer);
};

// ---- taco-coder ----

// freq.rs:103 FreqTable::from_weights. `starts` gets one u32 per symbol. Returns 0, or
// 1 (empty), 2 (too many symbols), 3 (bits > 32).
int from_weights(const uint64_t* w, size_t n, uint32_t bits, uint32_t* starts);

struct Interval {
    uint64_t start, freq;
    bool is_last;
};

// freq.rs:243 FreqTable::interval.
inline Interval table_interval(const uint32_t* starts, size_t n, uint32_t bits, size_t i) {
    uint64_t total = 1ULL << bits;
    uint64_t start = starts[i];
    if (i + 1 < n) return {start, (uint64_t)starts[i + 1] - start, false};
    return {start, total - start, true};
}

// freq.rs:229 FreqTable::find: the largest i with starts[i] <= target.
size_t table_find(const uint32_t* starts, size_t n, uint64_t target);

// ---- the weight step of the logs-profile mixer (crates/taco-match/src/mixer.rs) ----

// The table word of an input without a prediction and of a plain input
// (crates/hardshell-cuda/src/mixed.rs:31,104).
constexpr uint32_t MIX_NONE = 0xFFFFFFFFu;
constexpr uint32_t MIX_PLAIN = 0xFFFFFFFEu;

// Pass 1 of Mixer::mix (mixer.rs:276-287): W = sum(w) (a u128 there; below 2^64 for GPT-2
// weights, and the caller checks), w[p], and the top token (the first largest weight, 0 if every
// weight is 0). Returns 0, or 1 if p >= n, or 2 if the sum is 2^64 or more.
int mix_stats(const uint64_t* w, size_t n, uint32_t p, uint64_t* total, uint64_t* wp, uint32_t* top);

// The weights of Mixer::mix for the prediction p and the mixer probability q (units of 2^-16):
// p = MIX_NONE gives max(1, w) (mixer.rs:265-269, rule 1), p = MIX_PLAIN the weights unchanged
// (the table of GPT-2 alone), a token p the weights of apply (mixer.rs:491-516). Returns 0, or
// 1 if p is neither a token nor a table word, 2 if the sum is 2^64 or more, 3 if q is not in
// 1..=65535 (the reference's mix_record check, crates/hardshell-cuda/src/mixed.rs:71-73).
int mix_weights(const uint64_t* w, size_t n, uint32_t p, uint32_t q, uint64_t* out);

// encoder.rs:13 Encoder: the LZMA-style range encoder with a 64-bit window.
struct Encoder {
    unsigned __int128 low = 0;
    uint64_t range = ~0ULL;
    uint8_t cache = 0;
    size_t pending = 0;
    std::vector<uint8_t> out;
    size_t nonzero_len = 0;

    void encode_parts(uint64_t start, uint64_t freq, bool is_last, uint32_t bits);  // encoder.rs:98
    void encode_bit(uint32_t p1, bool bit);                                         // encoder.rs:113
    std::vector<uint8_t> finish();                                                  // encoder.rs:134
    size_t min_final_len() const { return nonzero_len; }

   private:
    void renormalise();  // encoder.rs:171
    void shift_low();    // encoder.rs:181
};

// decoder.rs:12 Decoder.
struct Decoder {
    const uint8_t* input = nullptr;
    size_t len = 0, pos = 0;
    uint64_t code = 0;
    uint64_t range = ~0ULL;

    Decoder(const uint8_t* in, size_t n);                                         // decoder.rs:30
    uint64_t target(uint32_t bits) const;                                         // decoder.rs:66
    bool decode_interval(uint64_t start, uint64_t freq, bool is_last, uint32_t bits);  // decoder.rs:80
    uint32_t decode_table(const uint32_t* starts, size_t n, uint32_t bits);       // decoder.rs:43
    bool decode_bit(uint32_t p1);                                                 // decoder.rs:103

   private:
    void renormalise();
    uint8_t next_byte() { return pos < len ? input[pos++] : 0; }
};

}  // namespace hso
