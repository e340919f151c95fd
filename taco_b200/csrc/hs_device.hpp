// The device-side layout of a loaded model and of the work buffers of one pass, shared by the
// kernels and the host runtime of the B200 HardShell backend.
#pragma once

#include <cstdint>

// The device error word (one int per device, 0 = no error): a bounded wait that gives up writes
// its wait's code (below 40); the coder op writes ERR_CODER_DIVISION when its frequency division
// is not exact after its correction steps; the prefill attention writes ERR_ATTN_SCRATCH when it
// is launched with more CTAs than scratch slots. The first code written stays.
constexpr int ERR_CODER_DIVISION = 40;
constexpr int ERR_ATTN_SCRATCH = 41;

namespace hs {

// Rows of the GEMM operand tiles and the padding of every K and N dimension.
constexpr int TILE_M = 128;
constexpr int TILE_N = 256;
constexpr int TILE_K = 128;
// Columns of one logits tile: the coder op reads the max of each tile (LOGIT_TILE columns; a
// model with a 16-bit ln_f uses tiles of LOGIT_TILE_WIDE columns).
constexpr int LOGIT_TILE = 128;
constexpr int LOGIT_TILE_WIDE = 64;
// The largest logit table the coder op keeps in shared memory (entries).
constexpr int MAX_LOGIT_TABLE = 16384;
// The largest vocabulary of the coder op (8 warps x 32 steps x 256 symbols).
constexpr int MAX_CODER_VOCAB = 65536;
// The largest context the attention kernels hold in shared memory (scores of one row).
constexpr int MAX_ATTN_CTX = 8192;

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

// One linear layer on the device: weights [Np, Kp] (K-major, zero padded), bias, multiplier.
struct LinearDev {
    const int8_t* w;
    int N, K, Np, Kp;
    const int32_t* b;
    const int32_t* m;
    int s;
};

struct LnDev {
    const int16_t* g;
    const int32_t* b;
    int32_t m;
    int s;
    int beta_frac;
};

struct LayerDev {
    LnDev ln1, ln2;
    LinearDev qkv, proj, fc, mlp;
    int32_t score_m;
    int score_s;
    int32_t out_m;
    int out_s;
    const int8_t* gelu;      // i8 outputs
    const int16_t* gelu16;   // i16 outputs (version 2), or null
    int gelu_off;            // 2^(b-1): the input range is [-off, off - 1]
};

// One row of a pass: the slot, the input token, the position, and the coder query
// (kind 0 = the interval of token `value`, 1 = the symbol that holds target `value`).
struct RowInfo {
    uint32_t slot, token, pos, kind;
    uint64_t value;
};

// The table words of the mixed coder op (crates/hardshell-cuda/src/mixed.rs:31,104): a row
// without a prediction (weights max(1, w)) and a plain row (the weights of GPT-2 alone).
constexpr uint32_t MIX_NONE = 0xFFFFFFFFu;
constexpr uint32_t MIX_PLAIN = 0xFFFFFFFEu;

// The mix record of one row (mixed.rs:60-90 mix_record): the table word p (a predicted token,
// MIX_NONE or MIX_PLAIN); for a token, the shift k, the factor m = 2^16 - q and the mixed
// weight wp = max(1, (R * q) >> k) of p. The weight of every other symbol is
// max(1, (w * m) >> k).
struct MixRow {
    uint32_t p, k, m, pad;
    uint64_t wp, pad2;
};

// The range decoder state of one coded block on the device (crates/taco-coder/src/decoder.rs
// Decoder: code, range, the next byte `pos` of its input payload[base .. base + len)), and
// whether an interval failed to hold its target.
struct DecState {
    uint64_t code, range, base, len, pos;
    uint32_t failed, pad;
};

// A run of up to 128 rows of one slot at consecutive positions pos0 .. pos0 + count - 1, whose
// rows are first_row .. first_row + count - 1 of the pass (the prefill attention unit).
struct AttnGroup {
    uint32_t first_row, count, slot, pos0;
};

// The epilogue of a GEMM tile: what happens to acc = W[n] . A[r] (exact s32).
enum EpiMode : int {
    EPI_ACT = 0,     // out8[r, n] = clamp(rescale(acc + b[n], m[n], s), -127, 127)
    EPI_GELU = 1,    // out8[r, n] = gelu[clamp(rescale(acc + b[n], m[n], s), lo, hi) + off]
    EPI_RESID = 2,   // x[r, n] = clamp(x[r, n] + rescale(acc + b[n], m[n], s), -R, R)
    EPI_LOGITS = 3,  // l = clamp(rescale(acc, m[n], s), +-2^40); tile max and d16 = min(tmax - l, last)
    EPI_RAW = 4,     // out32[r, n] = acc (the GEMM tests)
    EPI_DELTA = 5,   // out32[r, n] = clamp(rescale(acc + b[n], m[n], s), i32); the residual add and its
                     // clamp to [-R, R] happen in the next LayerNorm kernel: clamping the delta to the
                     // i32 range first gives the same result, because |x| <= R < 2^30.
    EPI_QKV = 6,     // as EPI_ACT; q (columns < d) to out8, k to the keys cache and v to the
                     // transposed values cache at the row's (slot, pos) (reference.rs:241-246)
    EPI_GELU16 = 7,  // as EPI_GELU with an i16 table (version 2 models): the output as two i8 planes,
                     // hi = floor(v / 256) to out8 and lo = (v mod 256) - 128 to out8_lo
};

struct EpiArgs {
    int R, N;
    const int32_t* b;
    const int32_t* m;
    int s;
    int8_t* out8;
    int ldo;
    const int8_t* gelu;
    int gelu_off;
    int32_t* x;
    int ldx;
    uint16_t* d16;
    int ldd;
    int64_t* tmax;
    int ldt;
    int last;
    int small;  // every rescaled output is below 2^30 in magnitude (host bound): 32-bit arithmetic
    // Version 2 (i16 activations as two i8 planes, v = 256 hi + lo + 128): the i16 GELU table and
    // the lo plane of EPI_GELU16, and for a GEMM over such planes the row sums of the weights
    // (the 128 * sum_k W[n][k] term of the recombination).
    const int16_t* gelu16;
    int8_t* out8_lo;
    const int64_t* wsum;
    int32_t* out32;
    // EPI_QKV: the rows of the pass and the caches of this layer.
    const RowInfo* rows;
    int8_t* kc;
    int8_t* vc;
    int L, layer, H, hd, n_ctx, d;
    // EPI_QKV on tensor cores: the v of the rows whose 32-row group is not a transposed run
    // (vt_run) goes here, row-major with stride ldv, for launch_v_scatter to place in vc.
    int8_t* vstage;
    int ldv;
    // EPI_QKV: whole 32 x 32-byte pieces of q, and of k and v for 32-row prefill runs, leave
    // through the TMA store maps that the launch passes (the batch made them).
    int kv_tma;
    // The first row of A that this launch reads (row tile mt reads A rows a_row0 + 128 mt ...);
    // the outputs are written from row 0. The LM head runs in row chunks with it.
    int a_row0;
};

// The 32 rows r0 .. r0 + 31 of a pass are one slot at 32 consecutive positions starting at a
// multiple of 16: their v is stored into the transposed values cache as 32-byte runs. The
// host form decides whether a pass needs launch_v_scatter; the device forms (the QKV epilogue
// and the scatter kernel) decide per group, with the same rule.
inline bool vt_run_host(const RowInfo* rows, int r0, int R, int n_ctx) {
    if (r0 + 31 >= R || (n_ctx & 15) != 0) return false;
    const RowInfo& a0 = rows[r0];
    if ((a0.pos & 15) != 0) return false;
    for (int i = 1; i < 32; i++)
        if (rows[r0 + i].slot != a0.slot || rows[r0 + i].pos != a0.pos + (uint32_t)i) return false;
    return true;
}

}  // namespace hs
