// The .hsm reader and the GPT-2 model loader of the B200 backend (host side), restated from crates/hardshell/src/hsm/reader.rs
// (HsmFile::parse, :357), hsm/header.rs (the JSON schema), hsm/merges.rs (the merges checks)
// and gpt2/model.rs (Model::load, :292; check_dims, :117).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace hsm {

struct RowRescale {
    std::vector<int32_t> m;
    uint32_t s = 0;
};

struct Linear {
    int rows = 0, cols = 0;
    std::vector<int8_t> w;  // [rows, cols]
    std::vector<int32_t> b;
    RowRescale rs;
};

struct LayerNormP {
    std::vector<int16_t> g;
    std::vector<int32_t> b;
    int32_t m = 0;
    uint32_t s = 0;
    uint32_t beta_frac = 0;
};

struct Block {
    LayerNormP ln_1, ln_2;
    Linear c_attn, c_proj, c_fc, mlp_proj;
    int32_t score_m = 0;
    uint32_t score_s = 0;
    int32_t out_m = 0;
    uint32_t out_s = 0;
    // The GELU table: 256 or 65536 entries, i8 outputs (wide = false) or i16 outputs.
    bool gelu_wide = false;
    std::vector<int8_t> gelu8;
    std::vector<int16_t> gelu16;
    int64_t gelu_offset = 0;  // 2^(b-1)
};

struct Model {
    uint32_t version = 1;
    int n_layer = 0, n_head = 0, d_model = 0, d_ff = 0, head_dim = 0, vocab = 0, n_ctx = 0;
    uint32_t eot = 0;
    uint32_t ln_k = 0, ln_j = 0;
    uint64_t ln_eps = 0;
    uint32_t softmax_p = 0;
    uint32_t ln_f_bits = 8;
    uint32_t ln_beta_frac = 0;
    std::vector<int8_t> wte;  // [vocab, d]
    RowRescale embed, logit;
    std::vector<int8_t> wpe;  // [n_ctx, d]
    RowRescale pos;
    std::vector<Block> blocks;
    LayerNormP ln_f;
    std::vector<int32_t> attn_exp;
    std::vector<uint64_t> logits_exp;
    // The vocabulary: bytes of each token; merges as (left, right) pairs in rank order.
    std::vector<uint8_t> vocab_bytes;
    std::vector<size_t> vocab_ends;
    std::vector<std::pair<uint32_t, uint32_t>> merges;

    bool is_wide() const;
};

// Parses and validates a full .hsm file. Returns false with a message on any error.
bool load_model(const uint8_t* bytes, size_t len, Model& out, std::string& err);

}  // namespace hsm
