// The unpacked .hsm model of the B200 backend, as the host reads it before the upload
// (hs_runtime.cu), the tokenizer builds on it (hs_tokenizer.cpp) and hs_model_check reports it.
// hsm_file.cpp fills it and refuses every file that hardshell::gpt2::Model::load refuses
// (crates/hardshell/src/gpt2/model.rs:292).
#pragma once

#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace hsm {

// Per-row fixed-point multipliers with one shift: y = rescale(x, m[row], s) (int.rs).
struct RowRescale {
    std::vector<int32_t> m;
    uint32_t s = 0;
};

// A linear layer: int8 weights [rows, cols] (row = output channel), i32 bias, per-row rescale.
struct Linear {
    int rows = 0, cols = 0;
    std::vector<int8_t> w;
    std::vector<int32_t> b;
    RowRescale rs;
};

// An integer LayerNorm: i16 gains, i32 betas (with beta_frac fractional bits in version 2),
// and one output rescale.
struct LayerNormP {
    std::vector<int16_t> g;
    std::vector<int32_t> b;
    int32_t m = 0;
    uint32_t s = 0;
    uint32_t beta_frac = 0;
};

// One transformer block. The GELU table maps a clamped fc output to the next activation: 256 or
// 65,536 entries centred on gelu_offset, i8 outputs, or i16 outputs (gelu_wide, version 2).
struct Block {
    LayerNormP ln_1, ln_2;
    Linear c_attn, c_proj, c_fc, mlp_proj;
    int32_t score_m = 0, out_m = 0;
    uint32_t score_s = 0, out_s = 0;
    bool gelu_wide = false;
    std::vector<int8_t> gelu8;
    std::vector<int16_t> gelu16;
    int64_t gelu_offset = 0;
};

struct Model {
    // Dimensions and constants of the header.
    uint32_t version = 1;
    int n_layer = 0, n_head = 0, d_model = 0, d_ff = 0, head_dim = 0, vocab = 0, n_ctx = 0;
    uint32_t eot = 0;
    uint32_t ln_k = 0, ln_j = 0, softmax_p = 0;
    uint64_t ln_eps = 0;
    uint32_t ln_f_bits = 8;     // 16 in a version 2 file with a 16-bit final LayerNorm
    uint32_t ln_beta_frac = 0;  // fractional bits of the LayerNorm betas (version 2)
    // Embeddings and the LM head (wte is both): [vocab, d] and [n_ctx, d] int8.
    std::vector<int8_t> wte, wpe;
    RowRescale embed, logit, pos;
    std::vector<Block> blocks;
    LayerNormP ln_f;
    // The exponent tables of the softmax and of the logits.
    std::vector<int32_t> attn_exp;
    std::vector<uint64_t> logits_exp;
    // The tokenizer's part: each token's bytes (vocab_bytes up to vocab_ends[id], from the end
    // of the token before) and the BPE merges (left, right) in rank order.
    std::vector<uint8_t> vocab_bytes;
    std::vector<size_t> vocab_ends;
    std::vector<std::pair<uint32_t, uint32_t>> merges;

    // A model with a part of format version 2 (16-bit activations somewhere).
    bool is_wide() const;
};

// Reads and checks a whole .hsm file into M; false with the reason in err if it is refused.
bool load_model(const uint8_t* bytes, size_t len, Model& M, std::string& err);

}  // namespace hsm
