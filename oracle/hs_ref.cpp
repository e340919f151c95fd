// TEST INFRASTRUCTURE ONLY (CPU oracle; see hs_int.hpp).
//
// The reference forward pass and the coder. Each function restates one reference function
// (file:line in the comment); the order of the integer steps is the reference's.
#include "hs_ref.hpp"

#include <algorithm>
#include <cstring>

#include "hs_int.hpp"

namespace hso {

static const int32_t RESIDUAL_LIMIT = (1 << 30) - 1;  // gpt2/mod.rs:113
static const int64_t SCORE_LIMIT = 1LL << 40;         // gpt2/mod.rs:116

// layernorm.rs:201-256.
void layernorm_apply(const Model& M, const LayerNormP& ln, const int32_t* x, int8_t* out8, int16_t* out16) {
    const int n = (int)ln.g.size();
    int64_t sum = 0;
    for (int i = 0; i < n; i++) sum += x[i];
    int64_t mean = floor_div(sum, n);
    u128 sum_sq = 0;
    for (int i = 0; i < n; i++) {
        int64_t dd = (int64_t)x[i] - mean;
        uint64_t d = dd < 0 ? (uint64_t)(-(i128)dd) : (uint64_t)dd;
        sum_sq += (u128)d * (u128)d;
    }
    u128 var = sum_sq / (u128)n;
    u128 root = isqrt_u128((var << (2 * M.ln_j)) + (u128)M.ln_eps);
    if (root < 1) root = 1;
    u128 inv_u = ((u128)1 << M.ln_k) / root;
    i128 inv = (i128)inv_u;
    for (int i = 0; i < n; i++) {
        i128 centred = (i128)((int64_t)x[i] - mean);
        i128 t = centred * inv * (i128)ln.g[i];
        i128 y;
        if (ln.beta_frac == 0) {
            y = rescale_wide(t, ln.m, ln.s) + (i128)ln.b[i];
        } else {
            i128 c = (i128)ln.b[i] << (ln.s - ln.beta_frac);
            y = rescale_wide_offset(t, ln.m, c, ln.s);
        }
        if (out16) out16[i] = clamp_act_i16(y);
        else out8[i] = clamp_act_i8(y);
    }
}

// softmax.rs:78-104.
bool softmax_ref(const int64_t* scores, size_t n, const std::vector<int32_t>& table, uint32_t p, int64_t* out) {
    if (p > 30 || n == 0) return false;
    int64_t mx = scores[0];
    for (size_t j = 1; j < n; j++) mx = std::max(mx, scores[j]);
    int64_t sum = 0;
    for (size_t j = 0; j < n; j++) {
        i128 d = (i128)mx - (i128)scores[j];
        int64_t idx = clamp_wide(d, 0, INT64_MAX);
        int64_t e = table_lookup(table.data(), table.size(), idx);
        out[j] = e;
        sum += e;
    }
    if (sum <= 0) sum = 1;
    for (size_t j = 0; j < n; j++) out[j] = floor_div(out[j] << p, sum);
    return true;
}

// logits.rs:62-72.
void logits_to_weights(const int64_t* logits, size_t n, const std::vector<uint64_t>& table, uint64_t* out) {
    int64_t mx = logits[0];
    for (size_t i = 1; i < n; i++) mx = std::max(mx, logits[i]);
    for (size_t i = 0; i < n; i++) {
        int64_t d = clamp_wide((i128)mx - (i128)logits[i], 0, INT64_MAX);
        out[i] = table_lookup(table.data(), table.size(), d);
    }
}

// kernels.rs:672 dot_i8 and :681 dot_i8_i16.
static inline int32_t dot_i8(const int8_t* a, const int8_t* b, int n) {
    int32_t s = 0;
    for (int i = 0; i < n; i++) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}
static inline int64_t dot_i8_i16(const int8_t* a, const int16_t* b, int n) {
    int64_t s = 0;
    for (int i = 0; i < n; i++) s += (int64_t)((int32_t)a[i] * (int32_t)b[i]);
    return s;
}

RefSession::RefSession(const Model* m, uint16_t k) : model(m), overlap(k) {
    const Model& M = *m;
    size_t cache = (size_t)M.n_layer * M.n_ctx * M.d_model;
    tokens.assign(M.n_ctx, 0);
    k_cache.assign(cache, 0);
    v_cache.assign(cache, 0);
    x.assign(M.d_model, 0);
    a.assign(M.d_model, 0);
    a16.assign(M.d_model, 0);
    qkv.assign(3 * M.d_model, 0);
    att.assign(M.d_model, 0);
    g.assign(M.d_ff, 0);
    g16.assign(M.d_ff, 0);
    scores.assign(M.n_ctx, 0);
    probs.assign(M.n_ctx, 0);
    head_acc.assign(M.head_dim, 0);
    logits.assign(M.vocab, 0);
    weights.assign(M.vocab, 0);
}

// reference.rs:144-162.
int RefSession::step(uint32_t token) {
    const Model& M = *model;
    if ((int)overlap + 2 > M.n_ctx) return 2;  // context.rs:113 check_overlap
    if (token >= (uint32_t)M.vocab) return 1;
    if (pos >= M.n_ctx) {
        int k = overlap;
        std::vector<uint32_t> kept(tokens.begin() + (M.n_ctx - k), tokens.begin() + M.n_ctx);
        reset();
        forward(M.eot, false);
        for (uint32_t t : kept) forward(t, false);
    }
    forward(token, true);
    return 0;
}

// reference.rs:170-205.
void RefSession::forward(uint32_t tok, bool want_logits) {
    const Model& M = *model;
    int t = pos;
    tokens[t] = tok;
    embed(tok, t);
    for (int l = 0; l < M.n_layer; l++) {
        attention(l, t);
        mlp(l);
    }
    if (!want_logits) {
        pos = t + 1;
        return;
    }
    const int d = M.d_model;
    if (M.ln_f_bits == 16) {
        layernorm_apply(M, M.ln_f, x.data(), nullptr, a16.data());
        for (int v = 0; v < M.vocab; v++) {
            int64_t s = dot_i8_i16(&M.wte[(size_t)v * d], a16.data(), d);
            logits[v] = clamp_wide(rescale(s, M.logit.m[v], M.logit.s), -SCORE_LIMIT, SCORE_LIMIT);
        }
    } else {
        layernorm_apply(M, M.ln_f, x.data(), a.data(), nullptr);
        for (int v = 0; v < M.vocab; v++) {
            int32_t s = dot_i8(&M.wte[(size_t)v * d], a.data(), d);
            logits[v] = clamp_wide(rescale(s, M.logit.m[v], M.logit.s), -SCORE_LIMIT, SCORE_LIMIT);
        }
    }
    logits_to_weights(logits.data(), M.vocab, M.logits_exp, weights.data());
    pos = t + 1;
}

// reference.rs:208-221.
void RefSession::embed(uint32_t tok, int t) {
    const Model& M = *model;
    const int d = M.d_model;
    const int8_t* te = &M.wte[(size_t)tok * d];
    const int8_t* pe = &M.wpe[(size_t)t * d];
    int32_t tm = M.embed.m[tok], pm = M.pos.m[t];
    for (int j = 0; j < d; j++) {
        i128 v = rescale(te[j], tm, M.embed.s) + rescale(pe[j], pm, M.pos.s);
        x[j] = clamp_i32(v, -RESIDUAL_LIMIT, RESIDUAL_LIMIT);
    }
}

// reference.rs:224-231 add_to_residual, with reference.rs:59 row_rescale.
static void add_to_residual(int32_t* x, const Linear& lin, const int8_t* input) {
    for (int r = 0; r < lin.rows; r++) {
        int32_t s = dot_i8(&lin.w[(size_t)r * lin.cols], input, lin.cols);
        i128 delta = rescale((int64_t)s + (int64_t)lin.b[r], lin.rs.m[r], lin.rs.s);
        x[r] = clamp_i32((i128)x[r] + delta, -RESIDUAL_LIMIT, RESIDUAL_LIMIT);
    }
}

// reference.rs:234-286.
void RefSession::attention(int layer, int t) {
    const Model& M = *model;
    const Block& B = M.blocks[layer];
    const int d = M.d_model, hd = M.head_dim;
    layernorm_apply(M, B.ln_1, x.data(), a.data(), nullptr);
    for (int r = 0; r < 3 * d; r++) {
        int32_t s = dot_i8(&B.c_attn.w[(size_t)r * d], a.data(), d);
        qkv[r] = clamp_act_i8(rescale((int64_t)s + (int64_t)B.c_attn.b[r], B.c_attn.rs.m[r], B.c_attn.rs.s));
    }
    size_t layer_base = (size_t)layer * M.n_ctx * d;
    size_t at = layer_base + (size_t)t * d;
    memcpy(&k_cache[at], &qkv[d], d);
    memcpy(&v_cache[at], &qkv[2 * d], d);
    int n = t + 1;
    for (int h = 0; h < M.n_head; h++) {
        int off = h * hd;
        const int8_t* q_h = &qkv[off];
        for (int j = 0; j < n; j++) {
            int32_t dot = dot_i8(q_h, &k_cache[layer_base + (size_t)j * d + off], hd);
            scores[j] = clamp_wide(rescale(dot, B.score_m, B.score_s), -SCORE_LIMIT, SCORE_LIMIT);
        }
        softmax_ref(scores.data(), n, M.attn_exp, M.softmax_p, probs.data());
        std::fill(head_acc.begin(), head_acc.end(), 0);
        for (int j = 0; j < n; j++) {
            int64_t p = probs[j];
            const int8_t* v_h = &v_cache[layer_base + (size_t)j * d + off];
            for (int c = 0; c < hd; c++) head_acc[c] += p * (int64_t)v_h[c];
        }
        for (int c = 0; c < hd; c++) att[off + c] = clamp_act_i8(rescale(head_acc[c], B.out_m, B.out_s));
    }
    add_to_residual(x.data(), B.c_proj, att.data());
}

// reference.rs:289-330.
void RefSession::mlp(int layer) {
    const Model& M = *model;
    const Block& B = M.blocks[layer];
    const int d = M.d_model, f = M.d_ff;
    layernorm_apply(M, B.ln_2, x.data(), a.data(), nullptr);
    int64_t lo = -B.gelu_offset, hi = B.gelu_offset - 1;
    for (int r = 0; r < f; r++) {
        int32_t s = dot_i8(&B.c_fc.w[(size_t)r * d], a.data(), d);
        int64_t in = clamp_wide(rescale((int64_t)s + (int64_t)B.c_fc.b[r], B.c_fc.rs.m[r], B.c_fc.rs.s), lo, hi);
        // gelu.rs:58 apply: clamp then look up at x + 2^(b-1).
        int64_t idx = clamp(in, lo, hi) + B.gelu_offset;
        if (B.gelu_wide) g16[r] = table_lookup(B.gelu16.data(), B.gelu16.size(), idx);
        else g[r] = table_lookup(B.gelu8.data(), B.gelu8.size(), idx);
    }
    if (!B.gelu_wide) {
        add_to_residual(x.data(), B.mlp_proj, g.data());
        return;
    }
    const Linear& lin = B.mlp_proj;
    for (int r = 0; r < d; r++) {
        int64_t s = dot_i8_i16(&lin.w[(size_t)r * f], g16.data(), f);
        i128 delta = rescale(s + (int64_t)lin.b[r], lin.rs.m[r], lin.rs.s);
        x[r] = clamp_i32((i128)x[r] + delta, -RESIDUAL_LIMIT, RESIDUAL_LIMIT);
    }
}

// ---- taco-coder ----

// freq.rs:103-157.
int from_weights(const uint64_t* w, size_t n, uint32_t bits, uint32_t* starts) {
    if (bits > 32) return 3;
    uint64_t total = 1ULL << bits;
    if (n == 0) return 1;
    if ((uint64_t)n > total) return 2;
    uint64_t symbols = n;
    u128 weight_sum = 0;
    size_t largest = 0;
    uint64_t largest_weight = 0;
    for (size_t i = 0; i < n; i++) {
        weight_sum += w[i];
        if (w[i] > largest_weight) {
            largest = i;
            largest_weight = w[i];
        }
    }
    bool all_zero = weight_sum == 0;
    if (all_zero) weight_sum = symbols;
    u128 spare = total - symbols;
    uint64_t acc = 0;
    for (size_t i = 0; i < n; i++) {
        u128 wi = all_zero ? 1 : w[i];
        uint64_t q = (uint64_t)(wi * spare / weight_sum);
        starts[i] = (uint32_t)acc;
        acc += 1 + q;
    }
    uint32_t remainder = (uint32_t)(total - acc);
    if (remainder > 0)
        for (size_t i = largest + 1; i < n; i++) starts[i] += remainder;
    return 0;
}

size_t table_find(const uint32_t* starts, size_t n, uint64_t target) {
    // partition_point(|s| s <= target) - 1
    size_t lo = 0, hi = n;
    while (lo < hi) {
        size_t mid = lo + (hi - lo) / 2;
        if ((uint64_t)starts[mid] <= target) lo = mid + 1;
        else hi = mid;
    }
    return lo - 1;
}

static const uint64_t TOP = 1ULL << 56;  // lib.rs:137

void Encoder::encode_parts(uint64_t start, uint64_t freq, bool is_last, uint32_t bits) {
    uint64_t r = range >> bits;
    uint64_t offset = r * start;
    low += offset;
    range = is_last ? range - offset : r * freq;
    renormalise();
}

void Encoder::encode_bit(uint32_t p1, bool bit) {
    uint64_t bound = (range >> 12) * (uint64_t)p1;
    if (bit) {
        range = bound;
    } else {
        low += bound;
        range -= bound;
    }
    renormalise();
}

void Encoder::renormalise() {
    while (range < TOP) {
        range <<= 8;
        shift_low();
    }
}

void Encoder::shift_low() {
    uint8_t carry = (uint8_t)((low >> 64) & 1);
    uint64_t window = (uint64_t)low;
    if (pending == 0 || window < 0xFF00000000000000ULL || carry != 0) {
        if (pending > 0) {
            uint8_t first = (uint8_t)(cache + carry);
            out.push_back(first);
            if (first != 0) nonzero_len = out.size();
            uint8_t fill = (uint8_t)(0xFF + carry);
            for (size_t i = 0; i + 1 < pending; i++) out.push_back(fill);
            if (fill != 0 && pending > 1) nonzero_len = out.size();
        }
        cache = (uint8_t)(window >> 56);
        pending = 0;
    }
    pending += 1;
    low = (unsigned __int128)(window << 8);
}

std::vector<uint8_t> Encoder::finish() {
    unsigned __int128 end = low + range;
    for (uint32_t k : {64u, 56u}) {
        unsigned __int128 mask = ((unsigned __int128)1 << k) - 1;
        unsigned __int128 v = (low + mask) & ~mask;
        if (v < end) {
            low = v;
            break;
        }
    }
    shift_low();
    shift_low();
    while (!out.empty() && out.back() == 0) out.pop_back();
    return out;
}

Decoder::Decoder(const uint8_t* in, size_t n) : input(in), len(n) {
    for (int i = 0; i < 8; i++) code = (code << 8) | next_byte();
}

uint64_t Decoder::target(uint32_t bits) const {
    uint64_t r = range >> bits;
    uint64_t total = 1ULL << bits;
    uint64_t t = code / r;
    return t < total - 1 ? t : total - 1;
}

bool Decoder::decode_interval(uint64_t start, uint64_t freq, bool is_last, uint32_t bits) {
    uint64_t t = target(bits);
    if (!(t >= start && t - start < freq)) return false;
    uint64_t r = range >> bits;
    uint64_t offset = r * start;
    code -= offset;
    range = is_last ? range - offset : r * freq;
    renormalise();
    return true;
}

uint32_t Decoder::decode_table(const uint32_t* starts, size_t n, uint32_t bits) {
    uint64_t r = range >> bits;
    uint64_t total = 1ULL << bits;
    uint64_t t = code / r;
    if (t > total - 1) t = total - 1;
    size_t i = table_find(starts, n, t);
    Interval iv = table_interval(starts, n, bits, i);
    uint64_t offset = r * iv.start;
    code -= offset;
    range = iv.is_last ? range - offset : r * iv.freq;
    renormalise();
    return (uint32_t)i;
}

bool Decoder::decode_bit(uint32_t p1) {
    uint64_t bound = (range >> 12) * (uint64_t)p1;
    bool bit = code < bound;
    if (bit) {
        range = bound;
    } else {
        code -= bound;
        range -= bound;
    }
    renormalise();
    return bit;
}

void Decoder::renormalise() {
    while (range < TOP) {
        range <<= 8;
        code = (code << 8) | next_byte();
    }
}

// ---- mixer.rs ----

int mix_stats(const uint64_t* w, size_t n, uint32_t p, uint64_t* total, uint64_t* wp, uint32_t* top) {
    if ((size_t)p >= n) return 1;
    u128 sum = 0;
    size_t t = 0;
    uint64_t tw = 0;
    for (size_t i = 0; i < n; i++) {
        sum += w[i];
        if (w[i] > tw) {  // the first largest weight; token 0 if every weight is 0
            t = i;
            tw = w[i];
        }
    }
    if (sum >> 64) return 2;
    *total = (uint64_t)sum;
    *wp = w[p];
    *top = (uint32_t)t;
    return 0;
}

int mix_weights(const uint64_t* w, size_t n, uint32_t p, uint32_t q, uint64_t* out) {
    if (p == MIX_PLAIN) {
        for (size_t i = 0; i < n; i++) out[i] = w[i];
        return 0;
    }
    if (p == MIX_NONE) {
        for (size_t i = 0; i < n; i++) out[i] = w[i] > 1 ? w[i] : 1;
        return 0;
    }
    if (q == 0 || q >= 65536) return 3;
    uint64_t total, wp;
    uint32_t top;
    int rc = mix_stats(w, n, p, &total, &wp, &top);
    if (rc) return rc;
    // apply (mixer.rs:491-516): R = max(W - w[p], 1), m = 2^16 - q, k = max(0, bitlen(R) + 16 - 62),
    // w'[i] = max(1, (w[i] * m) >> k), then w'[p] = max(1, (R * q) >> k). In u128 throughout: the
    // reference's u64 loop for weights below 2^48 gives the same values.
    const u128 r = total - wp > 0 ? (u128)(total - wp) : (u128)1;
    const u128 m = 65536u - q;
    int bits = 0;
    while (bits < 128 && (r >> bits) != 0) bits++;
    const int k = bits + 16 > 62 ? bits + 16 - 62 : 0;
    for (size_t i = 0; i < n; i++) {
        u128 x = ((u128)w[i] * m) >> k;
        out[i] = x > 1 ? (uint64_t)x : 1;  // below 2^62: w[i] <= R for i != p
    }
    u128 x = (r * q) >> k;
    out[p] = x > 1 ? (uint64_t)x : 1;
    return 0;
}

}  // namespace hso
