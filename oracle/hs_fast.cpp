// TEST INFRASTRUCTURE ONLY (CPU oracle; see hs_int.hpp and hs_fast.hpp).
#include "hs_fast.hpp"

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <thread>

#include "hs_int.hpp"
#include "hs_ref.hpp"

namespace hso {

namespace {

const int CHUNK = 32;  // crates/taco/src/fold.rs:24 FOLD_CHUNK
const size_t MIN_LANES = 4, MAX_LANES = 8;  // crates/taco/src/unfold.rs:249-256
const int32_t RES = (1 << 30) - 1;
const int64_t SCORE_LIMIT = 1LL << 40;

// kernels/fast.rs:27 (AVX2): sign-extend to i16 and multiply-add pairs into i32 lanes.
__attribute__((target("avx2"))) int32_t dot_i8_avx2(const int8_t* a, const int8_t* b, int n) {
    __m256i acc = _mm256_setzero_si256();
    int i = 0;
    for (; i + 16 <= n; i += 16) {
        __m256i x = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a + i)));
        __m256i y = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(b + i)));
        acc = _mm256_add_epi32(acc, _mm256_madd_epi16(x, y));
    }
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(acc), _mm256_extracti128_si256(acc, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
    int32_t r = _mm_cvtsi128_si32(s);
    for (; i < n; i++) r += (int32_t)a[i] * (int32_t)b[i];
    return r;
}

int32_t dot_i8_scalar(const int8_t* a, const int8_t* b, int n) {
    int32_t r = 0;
    for (int i = 0; i < n; i++) r += (int32_t)a[i] * (int32_t)b[i];
    return r;
}

bool have_avx2() {
    static int v = -1;
    if (v < 0) v = __builtin_cpu_supports("avx2") ? 1 : 0;
    return v == 1;
}

inline int32_t dot_i8(const int8_t* a, const int8_t* b, int n) {
    return have_avx2() ? dot_i8_avx2(a, b, n) : dot_i8_scalar(a, b, n);
}

int64_t dot_i8_i16(const int8_t* a, const int16_t* b, int n) {
    int64_t s = 0;
    for (int i = 0; i < n; i++) s += (int64_t)((int32_t)a[i] * (int32_t)b[i]);
    return s;
}

// out[r][n] = W[n] . A[r] for c rows: each weight row is read once for the chunk.
void matmul(const int8_t* W, int N, int K, const int8_t* A, int c, int32_t* out) {
    for (int n = 0; n < N; n++) {
        const int8_t* w = W + (size_t)n * K;
        for (int r = 0; r < c; r++) out[(size_t)r * N + n] = dot_i8(w, A + (size_t)r * K, K);
    }
}

// attention.rs:36 digits: four balanced base-256 digits of 0 <= p <= 2^30.
inline void digits(int64_t p, int8_t* d) {
    int64_t rest = p;
    for (int k = 0; k < 4; k++) {
        int64_t digit = ((rest + 128) & 255) - 128;
        d[k] = (int8_t)digit;
        rest = (rest - digit) >> 8;
    }
}

struct Row {
    int pos;
    uint32_t tok;
    long input;  // -1 for a restart row
    int slot;
};

struct Work {
    std::vector<int32_t> x, acc;
    std::vector<int8_t> a, qkv, att, g;
    std::vector<int16_t> a16, g16;
    std::vector<int64_t> acc64, scores, probs, logits;
    std::vector<int8_t> dig;  // [4, n_ctx]
    std::vector<uint64_t> w;
    std::vector<uint32_t> starts;
};

}  // namespace

FastBatch::FastBatch(const Model* m, int s, uint16_t k) : M(m), slots(s), overlap(k) {
    pos.assign(s, 0);
    hist.assign((size_t)s * m->n_ctx, 0);
    size_t per = (size_t)m->n_layer * m->n_ctx * m->d_model;
    kc.assign(per * s, 0);
    vt.assign(per * s, 0);
}

// The rows of a chunk: up to CHUNK rows of one slot at consecutive positions (prefill), or one row
// of each of up to MAX_LANES slots (lockstep lanes). Row r reads and writes the KV cache of its
// slot, at kc_all / vt_all + per * rows[r].slot.
static void run_chunk(const Model& M, int8_t* kc_all, int8_t* vt_all, size_t per, const Row* rows, int c, Work& w,
                      uint32_t bits, const uint32_t* kind, const uint64_t* value, uint64_t* answers,
                      uint64_t* weights, int* err) {
    const int d = M.d_model, f = M.d_ff, H = M.n_head, hd = M.head_dim, C = M.n_ctx, V = M.vocab;
    // ops.rs:52 embed
    for (int r = 0; r < c; r++) {
        const int8_t* te = &M.wte[(size_t)rows[r].tok * d];
        const int8_t* pe = &M.wpe[(size_t)rows[r].pos * d];
        int32_t tm = M.embed.m[rows[r].tok], pm = M.pos.m[rows[r].pos];
        for (int j = 0; j < d; j++) {
            i128 v = rescale(te[j], tm, M.embed.s) + rescale(pe[j], pm, M.pos.s);
            w.x[(size_t)r * d + j] = clamp_i32(v, -RES, RES);
        }
    }
    for (int l = 0; l < M.n_layer; l++) {
        const Block& B = M.blocks[l];
        for (int r = 0; r < c; r++) layernorm_apply(M, B.ln_1, &w.x[(size_t)r * d], &w.a[(size_t)r * d], nullptr);
        matmul(B.c_attn.w.data(), 3 * d, d, w.a.data(), c, w.acc.data());
        for (int r = 0; r < c; r++)
            for (int n = 0; n < 3 * d; n++) {
                int64_t v = (int64_t)w.acc[(size_t)r * 3 * d + n] + B.c_attn.b[n];
                w.qkv[(size_t)r * 3 * d + n] = clamp_act_i8(rescale(v, B.c_attn.rs.m[n], B.c_attn.rs.s));
            }
        size_t lbase = (size_t)l * H * C * hd;
        // attention.rs:138 write the keys and values of all rows of the chunk.
        for (int r = 0; r < c; r++) {
            int p = rows[r].pos;
            int8_t* kc = kc_all + per * rows[r].slot;
            int8_t* vt = vt_all + per * rows[r].slot;
            for (int h = 0; h < H; h++) {
                const int8_t* kk = &w.qkv[(size_t)r * 3 * d + d + h * hd];
                const int8_t* vv = &w.qkv[(size_t)r * 3 * d + 2 * d + h * hd];
                memcpy(kc + lbase + ((size_t)h * C + p) * hd, kk, hd);
                for (int ch = 0; ch < hd; ch++) vt[lbase + ((size_t)h * hd + ch) * C + p] = vv[ch];
            }
        }
        for (int r = 0; r < c; r++) {
            int n = rows[r].pos + 1;
            const int8_t* kc = kc_all + per * rows[r].slot;
            const int8_t* vt = vt_all + per * rows[r].slot;
            for (int h = 0; h < H; h++) {
                const int8_t* q = &w.qkv[(size_t)r * 3 * d + h * hd];
                const int8_t* keys = kc + lbase + (size_t)h * C * hd;
                int64_t mx = INT64_MIN;
                for (int j = 0; j < n; j++) {
                    int32_t dot = dot_i8(q, keys + (size_t)j * hd, hd);
                    int64_t sc = clamp_wide(rescale(dot, B.score_m, B.score_s), -SCORE_LIMIT, SCORE_LIMIT);
                    w.scores[j] = sc;
                    mx = std::max(mx, sc);
                }
                // attention.rs:233 softmax_fast.
                const int64_t last = (int64_t)M.attn_exp.size() - 1;
                uint64_t sum = 0;
                for (int j = 0; j < n; j++) {
                    int64_t dd = std::min(mx - w.scores[j], last);
                    uint64_t e = (uint64_t)M.attn_exp[dd];
                    w.probs[j] = (int64_t)e;
                    sum += e;
                }
                if (sum == 0) sum = 1;
                for (int j = 0; j < n; j++) {
                    int64_t p = (int64_t)(((uint64_t)w.probs[j] << M.softmax_p) / sum);
                    int8_t dg[4];
                    digits(p, dg);
                    for (int k = 0; k < 4; k++) w.dig[(size_t)k * C + j] = dg[k];
                }
                const int8_t* vals = vt + lbase + (size_t)h * hd * C;
                for (int ch = 0; ch < hd; ch++) {
                    int64_t acc = 0;
                    for (int k = 3; k >= 0; k--)
                        acc = (acc << 8) + dot_i8(&w.dig[(size_t)k * C], vals + (size_t)ch * C, n);
                    w.att[(size_t)r * d + h * hd + ch] = clamp_act_i8(rescale(acc, B.out_m, B.out_s));
                }
            }
        }
        // c_proj + residual (ops.rs:442, the same values as reference.rs:224).
        matmul(B.c_proj.w.data(), d, d, w.att.data(), c, w.acc.data());
        for (int r = 0; r < c; r++)
            for (int n = 0; n < d; n++) {
                int64_t v = (int64_t)w.acc[(size_t)r * d + n] + B.c_proj.b[n];
                i128 delta = rescale(v, B.c_proj.rs.m[n], B.c_proj.rs.s);
                int32_t& xv = w.x[(size_t)r * d + n];
                xv = clamp_i32((i128)xv + delta, -RES, RES);
            }
        for (int r = 0; r < c; r++) layernorm_apply(M, B.ln_2, &w.x[(size_t)r * d], &w.a[(size_t)r * d], nullptr);
        matmul(B.c_fc.w.data(), f, d, w.a.data(), c, w.acc.data());
        int64_t lo = -B.gelu_offset, hi = B.gelu_offset - 1;
        for (int r = 0; r < c; r++)
            for (int n = 0; n < f; n++) {
                int64_t v = (int64_t)w.acc[(size_t)r * f + n] + B.c_fc.b[n];
                int64_t in = clamp_wide(rescale(v, B.c_fc.rs.m[n], B.c_fc.rs.s), lo, hi);
                if (B.gelu_wide) w.g16[(size_t)r * f + n] = B.gelu16[in + B.gelu_offset];
                else w.g[(size_t)r * f + n] = B.gelu8[in + B.gelu_offset];
            }
        if (!B.gelu_wide) {
            matmul(B.mlp_proj.w.data(), d, f, w.g.data(), c, w.acc.data());
            for (int r = 0; r < c; r++)
                for (int n = 0; n < d; n++) {
                    int64_t v = (int64_t)w.acc[(size_t)r * d + n] + B.mlp_proj.b[n];
                    i128 delta = rescale(v, B.mlp_proj.rs.m[n], B.mlp_proj.rs.s);
                    int32_t& xv = w.x[(size_t)r * d + n];
                    xv = clamp_i32((i128)xv + delta, -RES, RES);
                }
        } else {
            for (int r = 0; r < c; r++)
                for (int n = 0; n < d; n++) {
                    int64_t s = dot_i8_i16(&B.mlp_proj.w[(size_t)n * f], &w.g16[(size_t)r * f], f);
                    i128 delta = rescale(s + (int64_t)B.mlp_proj.b[n], B.mlp_proj.rs.m[n], B.mlp_proj.rs.s);
                    int32_t& xv = w.x[(size_t)r * d + n];
                    xv = clamp_i32((i128)xv + delta, -RES, RES);
                }
        }
    }
    // ln_f, logits and the coder answer for the rows that answer an input.
    for (int r = 0; r < c; r++) {
        long in = rows[r].input;
        if (in < 0) continue;
        if (M.ln_f_bits == 16) {
            layernorm_apply(M, M.ln_f, &w.x[(size_t)r * d], nullptr, w.a16.data());
            for (int v = 0; v < V; v++) {
                int64_t s = dot_i8_i16(&M.wte[(size_t)v * d], w.a16.data(), d);
                w.logits[v] = clamp_wide(rescale(s, M.logit.m[v], M.logit.s), -SCORE_LIMIT, SCORE_LIMIT);
            }
        } else {
            layernorm_apply(M, M.ln_f, &w.x[(size_t)r * d], w.a.data(), nullptr);
            for (int v = 0; v < V; v++) {
                int32_t s = dot_i8(&M.wte[(size_t)v * d], w.a.data(), d);
                w.logits[v] = clamp_wide(rescale(s, M.logit.m[v], M.logit.s), -SCORE_LIMIT, SCORE_LIMIT);
            }
        }
        logits_to_weights(w.logits.data(), V, M.logits_exp, w.w.data());
        if (weights) memcpy(weights + (size_t)in * V, w.w.data(), (size_t)V * 8);
        if (answers) {
            from_weights(w.w.data(), V, bits, w.starts.data());
            size_t sym;
            if (kind[in] == 0) {
                sym = (size_t)value[in];
            } else {
                sym = table_find(w.starts.data(), V, value[in]);
            }
            Interval iv = table_interval(w.starts.data(), V, bits, sym);
            answers[3 * in] = sym;
            answers[3 * in + 1] = iv.start;
            answers[3 * in + 2] = iv.freq;
        }
    }
    (void)err;
}

int FastBatch::run(const uint32_t* slot, const uint32_t* token, size_t n, const uint32_t* kind, const uint64_t* value,
                   uint32_t bits, uint64_t* answers, uint64_t* weights, int threads, bool lanes) {
    const Model& m = *M;
    const int C = m.n_ctx;
    if (answers) {
        if (bits == 0 || bits > 32 || (uint64_t)m.vocab > (1ULL << bits)) return 5;
        for (size_t i = 0; i < n; i++) {
            if (kind[i] == 0 && value[i] >= (uint64_t)m.vocab) return 4;
            if (kind[i] == 1 && value[i] >= (1ULL << bits)) return 4;
            if (kind[i] > 1) return 4;
        }
    }
    for (size_t i = 0; i < n; i++) {
        if (slot[i] >= (uint32_t)slots) return 1;
        if (token[i] >= (uint32_t)m.vocab) return 2;
    }
    // Plan the rows of each slot (batch/plan.rs:60 with the restart of gpt2/context.rs).
    std::vector<std::vector<Row>> rows(slots);
    int k = std::min<int>(overlap, C - 2);
    for (size_t i = 0; i < n; i++) {
        int s = slot[i];
        uint32_t* h = &hist[(size_t)s * C];
        int at = pos[s];
        if (at >= C) {
            memmove(h + 1, h + (C - k), sizeof(uint32_t) * k);
            h[0] = m.eot;
            for (int q = 0; q <= k; q++) rows[s].push_back({q, h[q], -1, s});
            at = k + 1;
        }
        h[at] = token[i];
        rows[s].push_back({at, token[i], (long)i, s});
        pos[s] = at + 1;
    }
    std::vector<int> active;
    bool single = true;  // every active slot has one row: the step of a lockstep decode
    for (int s = 0; s < slots; s++)
        if (!rows[s].empty()) {
            active.push_back(s);
            single = single && rows[s].size() == 1;
        }
    // Lockstep lanes (crates/taco/src/unfold.rs:215-246 decode_blocks on the CPU): the slots go in
    // groups of ceil(slots / threads) clamped to [min(MIN_LANES, slots), MAX_LANES], and one thread
    // runs a group's rows as one chunk, so each weight row is read once for the group. Without
    // lanes (or with more than one row in a slot: a prefill), each slot is one task.
    std::vector<std::vector<Row>> groups;
    if (lanes && single && !active.empty()) {
        const size_t nt = (size_t)std::max(1, threads);
        const size_t fill = std::min<size_t>(active.size(), MIN_LANES);
        const size_t gs = std::min<size_t>(std::max((active.size() + nt - 1) / nt, fill), MAX_LANES);
        for (size_t g = 0; g < active.size(); g += gs) {
            groups.emplace_back();
            for (size_t k2 = g; k2 < std::min(active.size(), g + gs); k2++) groups.back().push_back(rows[active[k2]][0]);
        }
    }
    std::atomic<size_t> next(0);
    auto worker = [&]() {
        const int d = m.d_model, f = m.d_ff;
        Work w;
        size_t accn = std::max({(size_t)3 * d, (size_t)f, (size_t)d});
        w.x.assign((size_t)CHUNK * d, 0);
        w.acc.assign((size_t)CHUNK * accn, 0);
        w.a.assign((size_t)CHUNK * d, 0);
        w.a16.assign(d, 0);
        w.qkv.assign((size_t)CHUNK * 3 * d, 0);
        w.att.assign((size_t)CHUNK * d, 0);
        w.g.assign((size_t)CHUNK * f, 0);
        w.g16.assign((size_t)CHUNK * f, 0);
        w.scores.assign(C, 0);
        w.probs.assign(C, 0);
        w.dig.assign((size_t)4 * C, 0);
        w.logits.assign(m.vocab, 0);
        w.w.assign(m.vocab, 0);
        w.starts.assign(m.vocab, 0);
        size_t per = (size_t)m.n_layer * C * d;
        int err = 0;
        if (!groups.empty()) {
            for (size_t idx; (idx = next.fetch_add(1)) < groups.size();)
                run_chunk(m, kc.data(), vt.data(), per, groups[idx].data(), (int)groups[idx].size(), w, bits, kind,
                          value, answers, weights, &err);
            return;
        }
        while (true) {
            size_t idx = next.fetch_add(1);
            if (idx >= active.size()) break;
            int s = active[idx];
            const std::vector<Row>& rs = rows[s];
            size_t i = 0;
            while (i < rs.size()) {
                // A chunk: at most CHUNK rows at consecutive positions (a restart starts a new one).
                size_t j = i + 1;
                while (j < rs.size() && (int)(j - i) < CHUNK && rs[j].pos == rs[j - 1].pos + 1) j++;
                run_chunk(m, kc.data(), vt.data(), per, &rs[i], (int)(j - i), w, bits, kind, value, answers,
                          weights, &err);
                i = j;
            }
        }
    };
    int nt = std::max(1, std::min<int>(threads, (int)(groups.empty() ? active.size() : groups.size())));
    std::vector<std::thread> pool;
    for (int t = 1; t < nt; t++) pool.emplace_back(worker);
    worker();
    for (auto& t : pool) t.join();
    return 0;
}

}  // namespace hso

extern "C" {

void* hso_fast_new(void* model, int slots, uint16_t overlap) {
    return new hso::FastBatch((const hso::Model*)model, slots, overlap);
}
void hso_fast_free(void* b) { delete (hso::FastBatch*)b; }
void hso_fast_reset(void* b, int slot) { ((hso::FastBatch*)b)->pos[slot] = 0; }
int hso_fast_position(void* b, int slot) { return ((hso::FastBatch*)b)->pos[slot]; }
int hso_fast_run(void* b, const uint32_t* slot, const uint32_t* token, size_t n, const uint32_t* kind,
                 const uint64_t* value, uint32_t bits, uint64_t* answers, uint64_t* weights, int threads) {
    return ((hso::FastBatch*)b)->run(slot, token, n, kind, value, bits, answers, weights, threads, false);
}
// The same with lockstep lanes for decode steps (one row per slot).
int hso_fast_run_lanes(void* b, const uint32_t* slot, const uint32_t* token, size_t n, const uint32_t* kind,
                       const uint64_t* value, uint32_t bits, uint64_t* answers, uint64_t* weights, int threads) {
    return ((hso::FastBatch*)b)->run(slot, token, n, kind, value, bits, answers, weights, threads, true);
}

}  // extern "C"
