// TEST INFRASTRUCTURE ONLY (CPU oracle; see hs_int.hpp).
//
// The C interface of the oracle for the Python tests (ctypes), and the coded-block codec of
// crates/taco/src/codec.rs (encode_block :330, BlockDecoder :370-520) and payload.rs (varint).
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "hs_fast.hpp"
#include "hs_int.hpp"
#include "hs_model.hpp"
#include "hs_ref.hpp"

using namespace hso;

namespace {

void put_err(char* err, size_t cap, const std::string& m) {
    if (!err || cap == 0) return;
    size_t n = m.size() < cap - 1 ? m.size() : cap - 1;
    memcpy(err, m.data(), n);
    err[n] = 0;
}

// payload.rs:20 write_varint: minimal LEB128.
void write_varint(uint64_t v, std::vector<uint8_t>& out) {
    while (true) {
        uint8_t low = v & 0x7F;
        v >>= 7;
        if (v == 0) {
            out.push_back(low);
            return;
        }
        out.push_back(low | 0x80);
    }
}

// payload.rs:45 read_varint: minimal, at most 10 bytes, fits in u64.
bool read_varint(const uint8_t* b, size_t n, uint64_t& value, size_t& used) {
    value = 0;
    uint32_t shift = 0;
    for (size_t i = 0; i < n && i < 10; i++) {
        uint64_t group = b[i] & 0x7F;
        if (i == 9 && group > 1) return false;
        value |= group << shift;
        shift += 7;
        if ((b[i] & 0x80) == 0) {
            if (b[i] == 0 && i > 0) return false;
            used = i + 1;
            return true;
        }
    }
    return false;
}

}  // namespace

extern "C" {

void* hso_model_load(const uint8_t* bytes, size_t len, char* err, size_t errlen) {
    auto* m = new Model();
    std::string e;
    if (!load_model(bytes, len, *m, e)) {
        put_err(err, errlen, e);
        delete m;
        return nullptr;
    }
    return m;
}

void hso_model_free(void* m) { delete (Model*)m; }

// n_layer, n_head, d_model, d_ff, head_dim, vocab, n_ctx, eot, ln_f_bits, ln_beta_frac,
// is_wide, version, attn_exp_len, logits_exp_len, softmax_p, n_merges
void hso_model_dims(void* mp, int64_t* out) {
    Model& M = *(Model*)mp;
    int64_t v[16] = {M.n_layer, M.n_head, M.d_model, M.d_ff, M.head_dim, M.vocab, M.n_ctx, M.eot,
                     M.ln_f_bits, M.ln_beta_frac, M.is_wide(), M.version, (int64_t)M.attn_exp.size(),
                     (int64_t)M.logits_exp.size(), M.softmax_p, (int64_t)M.merges.size()};
    memcpy(out, v, sizeof(v));
}

int hso_vocab_token(void* mp, uint32_t id, const uint8_t** p, size_t* n) {
    Model& M = *(Model*)mp;
    if (id >= (uint32_t)M.vocab) return 1;
    size_t a = id ? M.vocab_ends[id - 1] : 0, b = M.vocab_ends[id];
    *p = M.vocab_bytes.data() + a;
    *n = b - a;
    return 0;
}

int hso_merges(void* mp, uint32_t* out, size_t cap) {
    Model& M = *(Model*)mp;
    size_t n = M.merges.size();
    for (size_t i = 0; i < n && 2 * i + 1 < cap; i++) {
        out[2 * i] = M.merges[i].first;
        out[2 * i + 1] = M.merges[i].second;
    }
    return (int)n;
}

void* hso_session_new(void* mp, uint16_t overlap) { return new RefSession((Model*)mp, overlap); }
void hso_session_free(void* s) { delete (RefSession*)s; }
void hso_session_reset(void* s) { ((RefSession*)s)->reset(); }
int hso_session_position(void* s) { return ((RefSession*)s)->pos; }

int hso_session_step(void* sp, uint32_t tok, uint64_t* weights) {
    RefSession& s = *(RefSession*)sp;
    int rc = s.step(tok);
    if (rc == 0 && weights) memcpy(weights, s.weights.data(), s.weights.size() * 8);
    return rc;
}

int hso_from_weights(const uint64_t* w, size_t n, uint32_t bits, uint32_t* starts) {
    return from_weights(w, n, bits, starts);
}

// out = {W, w[p], top} (mixer.rs:276-287).
int hso_mix_stats(const uint64_t* w, size_t n, uint32_t p, uint64_t* out) {
    uint32_t top = 0;
    int rc = mix_stats(w, n, p, &out[0], &out[1], &top);
    out[2] = top;
    return rc;
}

int hso_mix_weights(const uint64_t* w, size_t n, uint32_t p, uint32_t q, uint64_t* out) {
    return mix_weights(w, n, p, q, out);
}

// The answer of the coder op for one weight vector (lanes.rs:20 Query, batch.rs:463 run_coded):
// kind 0 = the interval of token `value`, kind 1 = the symbol whose interval holds `value`.
// out = {symbol, start, freq}. Returns 0, or the error code of from_weights, or 4 (bad query).
int hso_answer(const uint64_t* w, size_t n, uint32_t bits, uint32_t kind, uint64_t value, uint64_t* out) {
    std::vector<uint32_t> starts(n);
    int rc = from_weights(w, n, bits, starts.data());
    if (rc) return rc;
    uint64_t total = 1ULL << bits;
    size_t sym;
    if (kind == 0) {
        if (value >= n) return 4;
        sym = (size_t)value;
    } else {
        if (value >= total) return 4;
        sym = table_find(starts.data(), n, value);
    }
    Interval iv = table_interval(starts.data(), n, bits, sym);
    out[0] = sym;
    out[1] = iv.start;
    out[2] = iv.freq;
    return 0;
}

// One step of a session, then the answer of the coder op for its weights.
int hso_session_coded(void* sp, uint32_t tok, uint32_t kind, uint64_t value, uint32_t bits, uint64_t* out) {
    RefSession& s = *(RefSession*)sp;
    int rc = s.step(tok);
    if (rc) return 10 + rc;
    return hso_answer(s.weights.data(), s.weights.size(), bits, kind, value, out);
}

// codec.rs:330 encode_block without a stop (the stop only removes payloads that lose):
// start_block codes t[0]; the weights after t[i] code t[i+1]. payload = varint(n) || coder.
// Returns 0, or an error code; *out_len gets the payload length (also when cap is too small).
int hso_encode_block(void* mp, uint16_t overlap, const uint32_t* tokens, size_t n, uint8_t* out, size_t cap,
                     size_t* out_len) {
    Model& M = *(Model*)mp;
    RefSession s(&M, overlap);
    Encoder e;
    std::vector<uint32_t> starts(M.vocab);
    if (n > 0) {
        int rc = s.start_block();
        if (rc) return 10 + rc;
        for (size_t i = 0; i < n; i++) {
            if (i > 0) {
                rc = s.step(tokens[i - 1]);
                if (rc) return 10 + rc;
            }
            if (tokens[i] >= (uint32_t)M.vocab) return 4;
            from_weights(s.weights.data(), M.vocab, 32, starts.data());
            Interval iv = table_interval(starts.data(), M.vocab, 32, tokens[i]);
            e.encode_parts(iv.start, iv.freq, iv.is_last, 32);
        }
    }
    std::vector<uint8_t> payload;
    write_varint(n, payload);
    std::vector<uint8_t> coded = e.finish();
    payload.insert(payload.end(), coded.begin(), coded.end());
    *out_len = payload.size();
    if (payload.size() > cap) return 5;
    memcpy(out, payload.data(), payload.size());
    return 0;
}

// codec.rs:370-520 BlockDecoder with a new session (unfold.rs decode_group: BatchInput::Start).
// Returns 0, or 20 + reason for a corrupt block: 1 count, 2 token with no bytes, 3 tokens longer
// than the block, 4 tokens shorter than the block.
int hso_decode_block(void* mp, uint16_t overlap, const uint8_t* payload, size_t len, uint32_t original_len,
                     uint8_t* out, size_t cap, uint32_t* toks, size_t tok_cap, size_t* n_tokens) {
    Model& M = *(Model*)mp;
    uint64_t count;
    size_t used;
    if (!read_varint(payload, len, count, used)) return 21;
    if (count > original_len || count == 0) return 21;
    Decoder dec(payload + used, len - used);
    RefSession s(&M, overlap);
    int rc = s.start_block();
    if (rc) return 10 + rc;
    std::vector<uint32_t> starts(M.vocab);
    size_t out_len = 0;
    uint64_t done = 0;
    *n_tokens = 0;
    while (true) {
        from_weights(s.weights.data(), M.vocab, 32, starts.data());
        uint32_t tok = dec.decode_table(starts.data(), M.vocab, 32);
        size_t a = tok ? M.vocab_ends[tok - 1] : 0, b = M.vocab_ends[tok];
        if (tok == M.eot || a == b) return 22;
        if (b - a > original_len - out_len) return 23;
        if (out_len + (b - a) > cap) return 5;
        memcpy(out + out_len, M.vocab_bytes.data() + a, b - a);
        out_len += b - a;
        if (toks && done < tok_cap) toks[done] = tok;
        done += 1;
        *n_tokens = done;
        if (done >= count) break;
        rc = s.step(tok);
        if (rc) return 10 + rc;
    }
    if (out_len != original_len) return 24;
    return 0;
}

// ---- the range coder as objects (the coder golden test) ----

void* hso_enc_new() { return new Encoder(); }
void hso_enc_free(void* e) { delete (Encoder*)e; }
void hso_enc_interval(void* e, uint64_t start, uint64_t freq, int is_last, uint32_t bits) {
    ((Encoder*)e)->encode_parts(start, freq, is_last != 0, bits);
}
void hso_enc_bit(void* e, uint32_t p1, int bit) { ((Encoder*)e)->encode_bit(p1, bit != 0); }
size_t hso_enc_min_final_len(void* e) { return ((Encoder*)e)->min_final_len(); }
// Finishes the stream; the encoder can not be used again. Returns the length.
size_t hso_enc_finish(void* e, uint8_t* out, size_t cap) {
    std::vector<uint8_t> b = ((Encoder*)e)->finish();
    if (b.size() <= cap) memcpy(out, b.data(), b.size());
    return b.size();
}

struct DecBox {
    std::vector<uint8_t> bytes;
    std::unique_ptr<Decoder> d;
};
void* hso_dec_new(const uint8_t* in, size_t n) {
    auto* box = new DecBox();
    box->bytes.assign(in, in + n);
    box->d.reset(new Decoder(box->bytes.data(), n));
    return box;
}
void hso_dec_free(void* d) { delete (DecBox*)d; }
uint64_t hso_dec_target(void* d, uint32_t bits) { return ((DecBox*)d)->d->target(bits); }
int hso_dec_interval(void* d, uint64_t start, uint64_t freq, int is_last, uint32_t bits) {
    return ((DecBox*)d)->d->decode_interval(start, freq, is_last != 0, bits) ? 0 : 1;
}
uint32_t hso_dec_table(void* d, const uint32_t* starts, size_t n, uint32_t bits) {
    return ((DecBox*)d)->d->decode_table(starts, n, bits);
}
int hso_dec_bit(void* d, uint32_t p1) { return ((DecBox*)d)->d->decode_bit(p1) ? 1 : 0; }

// ---- op-level checkers for the GPU kernels ----

// layernorm.rs:201 for `rows` rows. which: 2*layer (ln_1), 2*layer+1 (ln_2), -1 (ln_f).
void hso_layernorm_rows(void* mp, int which, const int32_t* x, size_t rows, int8_t* out8, int16_t* out16) {
    Model& M = *(Model*)mp;
    const LayerNormP& ln = which < 0 ? M.ln_f : (which % 2 == 0 ? M.blocks[which / 2].ln_1 : M.blocks[which / 2].ln_2);
    for (size_t r = 0; r < rows; r++)
        layernorm_apply(M, ln, x + r * M.d_model, out8 ? out8 + r * M.d_model : nullptr,
                        out16 ? out16 + r * M.d_model : nullptr);
}

}  // extern "C"
