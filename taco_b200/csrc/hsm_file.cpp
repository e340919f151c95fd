// The .hsm model file of the B200 backend: read, validated and unpacked on the host. A file is
// accepted exactly when hardshell::gpt2::Model::load accepts it (crates/hardshell/src/gpt2/
// model.rs:292). The rules come from the reference; the structure here is this backend's own:
//
//   1. the preamble (magic, version, header length) and a UTF-8 header (hsm/reader.rs:357-380);
//   2. the header, read by a JSON reader that the schema drives: each object is a table of
//      fields with a handler each; unknown and repeated fields, non-integer numbers and wrong
//      kinds are refused as they are met (hsm/header.rs:15-200, deny_unknown_fields);
//   3. the model fields (check_config, check_version: hsm/reader.rs:270-320);
//   4. one walk over the sections in file order, each at the 64-byte boundary after the one
//      before, zero padding between, the file ending at the last one (hsm/reader.rs:382-440),
//      decoding the vocabulary (reader.rs:173-200) and the merges (hsm/merges.rs:66-120);
//   5. the GPT-2 tensor set as a list of specifications built from the dimensions, matched
//      against the file's tensor table by name (gpt2/model.rs:117-403).
#include "hsm_file.hpp"

#include <cstring>
#include <functional>
#include <string>
#include <unordered_map>
#include <unordered_set>

namespace hsm {

namespace {

bool fail(std::string& err, const std::string& why) {
    if (err.empty()) err = why;
    return false;
}

// ---- 1. UTF-8 (Unicode table 3-7): the header must be well-formed before it is parsed ----

bool utf8_ok(const uint8_t* p, size_t n) {
    size_t i = 0;
    while (i < n) {
        const uint8_t b = p[i];
        if (b < 0x80) {
            i++;
            continue;
        }
        int k;
        uint8_t lo = 0x80, hi = 0xBF;
        if (b >= 0xC2 && b <= 0xDF) k = 1;
        else if (b >= 0xE0 && b <= 0xEF) k = 2, lo = b == 0xE0 ? 0xA0 : 0x80, hi = b == 0xED ? 0x9F : 0xBF;
        else if (b >= 0xF0 && b <= 0xF4) k = 3, lo = b == 0xF0 ? 0x90 : 0x80, hi = b == 0xF4 ? 0x8F : 0xBF;
        else return false;
        if (n - i <= (size_t)k) return false;
        if (p[i + 1] < lo || p[i + 1] > hi) return false;
        for (int j = 2; j <= k; j++)
            if ((p[i + j] & 0xC0) != 0x80) return false;
        i += k + 1;
    }
    return true;
}

// ---- 2. the header: a JSON reader driven by the schema ----

// What a handler gets: the reader positioned at the field's value.
class Json;
using Handler = std::function<bool(Json&)>;

struct Field {
    const char* name;
    bool required;
    Handler read;
};

class Json {
  public:
    Json(const char* p, const char* end, std::string& err) : p_(p), end_(end), err_(err) {}

    bool bad(const std::string& why) { return fail(err_, "header JSON: " + why); }

    void space() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) p_++;
    }
    bool at_end() {
        space();
        return p_ == end_;
    }
    bool peek(char c) {
        space();
        return p_ < end_ && *p_ == c;
    }
    bool eat(char c) {
        if (!peek(c)) return false;
        p_++;
        return true;
    }

    // An unsigned integer literal (digits only, no leading zero, at most `max`).
    bool uint(uint64_t max, uint64_t& out, const std::string& what) {
        space();
        const char* s = p_;
        uint64_t v = 0;
        bool over = false;
        while (p_ < end_ && *p_ >= '0' && *p_ <= '9') {
            const uint64_t dgt = (uint64_t)(*p_ - '0');
            if (v > (UINT64_MAX - dgt) / 10) over = true;
            v = v * 10 + dgt;
            p_++;
        }
        if (p_ == s) return bad(what + " is not an unsigned integer");
        if (p_ - s > 1 && *s == '0') return bad(what + " has a leading zero");
        if (p_ < end_ && (*p_ == '.' || *p_ == 'e' || *p_ == 'E')) return bad(what + " is not an integer");
        if (over || v > max) return bad(what + " is out of range");
        out = v;
        return true;
    }

    // A string with the JSON escapes (a \u escape of a surrogate must pair).
    bool str(std::string& out, const std::string& what) {
        if (!eat('"')) return bad(what + " is not a string");
        out.clear();
        for (;;) {
            if (p_ >= end_) return bad("an unterminated string");
            const unsigned char c = (unsigned char)*p_++;
            if (c == '"') return true;
            if (c < 0x20) return bad("a control character in a string");
            if (c != '\\') {
                out.push_back((char)c);
                continue;
            }
            if (p_ >= end_) return bad("a truncated escape");
            const char e = *p_++;
            const char* simple = "\"\\/bfnrt";
            const char* mapped = "\"\\/\b\f\n\r\t";
            if (const char* at = strchr(simple, e); at && e) {
                out.push_back(mapped[at - simple]);
                continue;
            }
            if (e != 'u') return bad("an unknown escape");
            uint32_t cp;
            if (!hex4(cp)) return false;
            if (cp >= 0xDC00 && cp < 0xE000) return bad("a lone low surrogate");
            if (cp >= 0xD800 && cp < 0xDC00) {
                uint32_t low;
                if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return bad("a lone high surrogate");
                p_ += 2;
                if (!hex4(low) || low < 0xDC00 || low >= 0xE000) return bad("a bad surrogate pair");
                cp = 0x10000 + ((cp - 0xD800) << 10) + (low - 0xDC00);
            }
            utf8(cp, out);
        }
    }

    // An object whose fields are those of `schema`, each at most once; the required ones present.
    bool object(const std::vector<Field>& schema, const std::string& where) {
        if (!eat('{')) return bad(where + " is not an object");
        std::vector<char> seen(schema.size(), 0);
        if (!eat('}')) {
            do {
                std::string key;
                if (!str(key, "a field name of " + where)) return false;
                if (!eat(':')) return bad("':' expected after " + where + key.substr(0, 64));
                size_t k = 0;
                while (k < schema.size() && key != schema[k].name) k++;
                if (k == schema.size()) return bad("unknown field " + where + key.substr(0, 64));
                if (seen[k]) return bad("repeated field " + where + key);
                seen[k] = 1;
                if (!schema[k].read(*this)) return false;
            } while (eat(','));
            if (!eat('}')) return bad("',' or '}' expected in " + where);
        }
        for (size_t k = 0; k < schema.size(); k++)
            if (schema[k].required && !seen[k]) return bad("missing field " + where + schema[k].name);
        return true;
    }

    // An array: `item` reads each element.
    bool array(const std::function<bool(Json&)>& item, const std::string& where) {
        if (!eat('[')) return bad(where + " is not an array");
        if (eat(']')) return true;
        do {
            if (!item(*this)) return false;
        } while (eat(','));
        if (!eat(']')) return bad("',' or ']' expected in " + where);
        return true;
    }

  private:
    bool hex4(uint32_t& v) {
        if (end_ - p_ < 4) return bad("a truncated \\u escape");
        v = 0;
        for (int i = 0; i < 4; i++) {
            const char c = *p_++;
            const int h = c >= '0' && c <= '9' ? c - '0' : c >= 'a' && c <= 'f' ? c - 'a' + 10
                                                          : c >= 'A' && c <= 'F' ? c - 'A' + 10 : -1;
            if (h < 0) return bad("a bad \\u escape");
            v = v << 4 | (uint32_t)h;
        }
        return true;
    }
    static void utf8(uint32_t cp, std::string& o) {
        if (cp < 0x80) {
            o.push_back((char)cp);
            return;
        }
        const int n = cp < 0x800 ? 2 : cp < 0x10000 ? 3 : 4;
        const uint8_t lead[5] = {0, 0, 0xC0, 0xE0, 0xF0};
        o.push_back((char)(lead[n] | (cp >> (6 * (n - 1)))));
        for (int i = n - 2; i >= 0; i--) o.push_back((char)(0x80 | ((cp >> (6 * i)) & 0x3F)));
    }

    const char* p_;
    const char* end_;
    std::string& err_;
};

// The header's content.
struct TensorEntry {
    std::string name, dtype;
    std::vector<uint64_t> shape;
    uint64_t offset = 0, length = 0;
    bool has_shift = false;
    uint64_t shift = 0;
};

struct Header {
    std::string arch;
    uint64_t n_layer = 0, n_head = 0, d_model = 0, d_ff = 0, vocab = 0, n_ctx = 0, eot = 0;
    uint64_t ln_k = 0, ln_j = 0, ln_eps = 0, softmax_p = 0, ln_f_bits = 0, beta_frac = 0;
    bool has_lnf = false, has_bf = false;
    uint64_t voff = 0, vlen = 0, moff = 0, mlen = 0;
    bool has_merges = false;
    std::vector<TensorEntry> tensors;
};

constexpr uint64_t U32 = 0xFFFFFFFFull, U8 = 255, U64 = UINT64_MAX;

bool read_header(const char* p, const char* end, Header& h, std::string& err) {
    Json j(p, end, err);
    auto u = [](uint64_t max, uint64_t& dst, const char* what) {
        return [max, &dst, what](Json& r) { return r.uint(max, dst, what); };
    };
    auto flag_u = [](uint64_t max, uint64_t& dst, bool& has, const char* what) {
        return [max, &dst, &has, what](Json& r) {
            has = true;
            return r.uint(max, dst, what);
        };
    };
    const std::vector<Field> constants = {
        {"ln_k", true, u(U8, h.ln_k, "ln_k")},
        {"ln_j", true, u(U8, h.ln_j, "ln_j")},
        {"ln_eps", true, u(U64, h.ln_eps, "ln_eps")},
        {"softmax_p", true, u(U8, h.softmax_p, "softmax_p")},
        {"ln_f_bits", false, flag_u(U8, h.ln_f_bits, h.has_lnf, "ln_f_bits")},
        {"ln_beta_frac", false, flag_u(U8, h.beta_frac, h.has_bf, "ln_beta_frac")},
    };
    const std::vector<Field> model = {
        {"architecture", true, [&](Json& r) { return r.str(h.arch, "model.architecture"); }},
        {"n_layer", true, u(U32, h.n_layer, "n_layer")},
        {"n_head", true, u(U32, h.n_head, "n_head")},
        {"d_model", true, u(U32, h.d_model, "d_model")},
        {"d_ff", true, u(U32, h.d_ff, "d_ff")},
        {"vocab_size", true, u(U32, h.vocab, "vocab_size")},
        {"n_ctx", true, u(U32, h.n_ctx, "n_ctx")},
        {"eot_token", true, u(U32, h.eot, "eot_token")},
        {"constants", true, [&](Json& r) { return r.object(constants, "model.constants."); }},
    };
    const std::vector<Field> vocabulary = {{"offset", true, u(U64, h.voff, "vocabulary.offset")},
                                           {"length", true, u(U64, h.vlen, "vocabulary.length")}};
    const std::vector<Field> merges = {{"offset", true, u(U64, h.moff, "merges.offset")},
                                       {"length", true, u(U64, h.mlen, "merges.length")}};
    auto tensor = [&](Json& r) {
        TensorEntry t;
        const std::vector<Field> fields = {
            {"name", true, [&](Json& q) { return q.str(t.name, "tensors[].name"); }},
            {"dtype", true, [&](Json& q) { return q.str(t.dtype, "tensors[].dtype"); }},
            {"shape", true,
             [&](Json& q) {
                 return q.array(
                     [&](Json& e) {
                         uint64_t d;
                         if (!e.uint(U64, d, "a shape dimension")) return false;
                         t.shape.push_back(d);
                         return true;
                     },
                     "tensors[].shape");
             }},
            {"offset", true, u(U64, t.offset, "tensors[].offset")},
            {"length", true, u(U64, t.length, "tensors[].length")},
            {"shift", false, flag_u(U8, t.shift, t.has_shift, "tensors[].shift")},
        };
        if (!r.object(fields, "tensors[].")) return false;
        h.tensors.push_back(std::move(t));
        return true;
    };
    const std::vector<Field> top = {
        {"model", true, [&](Json& r) { return r.object(model, "model."); }},
        {"vocabulary", true, [&](Json& r) { return r.object(vocabulary, "vocabulary."); }},
        {"merges", false,
         [&](Json& r) {
             h.has_merges = true;
             return r.object(merges, "merges.");
         }},
        {"tensors", true, [&](Json& r) { return r.array(tensor, "tensors"); }},
    };
    if (!j.object(top, "")) return false;
    if (!j.at_end()) return j.bad("characters after the header object");
    return true;
}

// ---- 3. the model fields ----

// A name: 1 to 128 characters from a-z 0-9 _ . (hsm/header.rs).
bool good_name(const std::string& n) {
    if (n.empty() || n.size() > 128) return false;
    for (unsigned char c : n)
        if (!((c >= 'a' && c <= 'z') || (c >= '0' && c <= '9') || c == '_' || c == '.')) return false;
    return true;
}

bool check_fields(const Header& h, uint32_t version, std::string& err) {
    // check_config
    if (!good_name(h.arch)) return fail(err, "model.architecture: 1 to 128 characters from a-z 0-9 _ .");
    if (h.vocab == 0 || h.vocab > (1u << 20)) return fail(err, "model.vocab_size: out of 1..=2^20");
    if (h.eot >= h.vocab) return fail(err, "model.eot_token: not below vocab_size");
    if (h.ln_k > 48 || h.ln_j > 16) return fail(err, "model.constants: ln_k or ln_j out of range");
    if (h.ln_eps == 0 || h.ln_eps > (1ULL << 62)) return fail(err, "model.constants.ln_eps: out of 1..=2^62");
    if (h.softmax_p > 30) return fail(err, "model.constants.softmax_p: above 30");
    // check_version: version 2 exactly when the file has a part of version 2.
    if (h.has_lnf && h.ln_f_bits != 16) return fail(err, "model.constants.ln_f_bits: must be 16");
    if (h.has_bf && (h.beta_frac == 0 || h.beta_frac > 16)) return fail(err, "model.constants.ln_beta_frac: out of 1..=16");
    bool wide_gelu = false;
    for (const TensorEntry& t : h.tensors) {
        const std::string& n = t.name;
        wide_gelu |= t.dtype == "i16" && n.size() >= 9 && n.compare(n.size() - 9, 9, ".mlp.gelu") == 0;
    }
    if ((h.has_lnf || h.has_bf || wide_gelu ? 2u : 1u) != version)
        return fail(err, "version: 2 exactly when the file has ln_f_bits, ln_beta_frac or an i16 GELU table");
    // check_dims (gpt2/model.rs:117)
    if (h.arch != "gpt2") return fail(err, "model.architecture: only gpt2 is read");
    if (h.n_layer == 0 || h.n_layer > 1024) return fail(err, "model.n_layer: out of 1..=1024");
    if (h.d_model == 0 || h.d_model > 65536) return fail(err, "model.d_model: out of 1..=65536");
    if (h.d_ff == 0 || h.d_ff > 65536) return fail(err, "model.d_ff: out of 1..=65536");
    if (h.n_head == 0 || h.d_model % h.n_head) return fail(err, "model.n_head: must divide d_model");
    if (h.n_ctx < 2 || h.n_ctx > 65536) return fail(err, "model.n_ctx: out of 2..=65536");
    return true;
}

// ---- 4. the sections ----

uint64_t next64(uint64_t x) { return (x + 63) & ~(uint64_t)63; }

size_t width_of(const std::string& dtype) {
    return dtype == "i8" ? 1 : dtype == "i16" ? 2 : dtype == "i32" ? 4 : dtype == "u64" ? 8 : 0;
}

// The walk over the sections: each starts at next64 of the end of the one before, with zero bytes
// between; take() checks one section and moves past it.
class Sections {
  public:
    Sections(const uint8_t* f, size_t n, uint64_t start, std::string& err) : f_(f), n_(n), at_(start), err_(err) {}

    bool take(uint64_t offset, uint64_t length, const std::string& what, const uint8_t** data) {
        const uint64_t want = next64(at_);
        if (offset != want) return fail(err_, "layout: " + what + " is not at the 64-byte boundary after the section before");
        if (want > n_ || length > n_ - want) return fail(err_, "truncated: " + what + " runs past the end of the file");
        for (uint64_t i = at_; i < want; i++)
            if (f_[i]) return fail(err_, "non-zero padding at byte " + std::to_string(i));
        *data = f_ + want;
        at_ = want + length;
        return true;
    }
    bool at_end() const { return at_ == n_ ? true : fail(err_, "layout: bytes after the last section"); }

  private:
    const uint8_t* f_;
    size_t n_;
    uint64_t at_;
    std::string& err_;
};

bool read_vocabulary(const uint8_t* s, uint64_t len, uint64_t count, Model& M, std::string& err) {
    M.vocab_bytes.clear();
    M.vocab_ends.clear();
    M.vocab_ends.reserve(count);
    uint64_t at = 0;
    for (uint64_t t = 0; t < count; t++) {
        if (len - at < 2) return fail(err, "vocabulary: token " + std::to_string(t) + " has no length");
        const uint64_t l = (uint64_t)s[at] | (uint64_t)s[at + 1] << 8;
        at += 2;
        if (len - at < l) return fail(err, "vocabulary: token " + std::to_string(t) + " runs past the section");
        M.vocab_bytes.insert(M.vocab_bytes.end(), s + at, s + at + l);
        M.vocab_ends.push_back(M.vocab_bytes.size());
        at += l;
    }
    return at == len || fail(err, "vocabulary: bytes after the last token");
}

std::string token_of(const Model& M, uint32_t id) {
    const size_t a = id ? M.vocab_ends[id - 1] : 0;
    return std::string((const char*)M.vocab_bytes.data() + a, M.vocab_ends[id] - a);
}

bool read_merges(const uint8_t* s, uint64_t len, Model& M, std::string& err) {
    if (len == 0 || len % 8) return fail(err, "merges.length: a positive multiple of 8");
    // A byte string shared by two tokens can be no merge's result (merges.rs:81-88).
    std::unordered_map<std::string, int64_t> owner;
    for (uint32_t i = 0; i < (uint32_t)M.vocab_ends.size(); i++) {
        auto ins = owner.emplace(token_of(M, i), (int64_t)i);
        if (!ins.second) ins.first->second = -1;
    }
    std::unordered_set<uint64_t> pairs;
    const uint32_t V = (uint32_t)M.vocab_ends.size();
    for (uint64_t r = 0; r < len / 8; r++) {
        uint32_t a, b;
        memcpy(&a, s + 8 * r, 4);
        memcpy(&b, s + 8 * r + 4, 4);
        const std::string at = "merges[" + std::to_string(r) + "]: ";
        if (a >= V || b >= V) return fail(err, at + "an id is not in the vocabulary");
        const std::string left = token_of(M, a), right = token_of(M, b);
        if (left.empty() || right.empty()) return fail(err, at + "a part has no bytes");
        if (!pairs.insert((uint64_t)a << 32 | b).second) return fail(err, at + "the pair occurs two times");
        auto it = owner.find(left + right);
        if (it == owner.end() || it->second < 0) return fail(err, at + "the joined bytes are not one token's");
        M.merges.emplace_back(a, b);
    }
    return true;
}

// ---- 5. the GPT-2 tensors ----

struct Blob {
    const TensorEntry* e;
    const uint8_t* data;
    bool used = false;
};

template <typename T>
std::vector<T> le_vector(const uint8_t* p, uint64_t bytes) {
    std::vector<T> v(bytes / sizeof(T));
    if (bytes) memcpy(v.data(), p, bytes);  // the file is little-endian, as is the host (x86-64)
    return v;
}

// softmax.rs:60 is_valid_exp_table: not empty, first >= 1, entries >= 0, not increasing.
template <typename T>
bool exp_table_ok(const std::vector<T>& t) {
    if (t.empty() || t[0] < (T)1) return false;
    for (size_t i = 0; i < t.size(); i++)
        if (t[i] < (T)0 || (i && t[i] > t[i - 1])) return false;
    return true;
}

class TensorSet {
  public:
    TensorSet(std::unordered_map<std::string, Blob>& blobs, std::string& err) : blobs_(blobs), err_(err) {}

    // The tensor `name` with this dtype, this shape (empty: any one-dimensional shape) and a
    // shift exactly when `shift` says; marks it used.
    const Blob* get(const std::string& name, const char* dtype, const std::vector<uint64_t>& shape, bool shift) {
        auto it = blobs_.find(name);
        if (it == blobs_.end() || it->second.used) {
            fail(err_, "missing tensor " + name);
            return nullptr;
        }
        const TensorEntry& e = *it->second.e;
        const bool shape_ok = shape.empty() ? e.shape.size() == 1 : e.shape == shape;
        if (!shape_ok) return fail(err_, "tensor " + name + ": not the shape the model needs"), nullptr;
        if (e.dtype != dtype) return fail(err_, "tensor " + name + ": not the dtype the model needs"), nullptr;
        if (e.has_shift != shift)
            return fail(err_, "tensor " + name + (shift ? ": a rescale needs a shift" : ": has a shift")), nullptr;
        it->second.used = true;
        return &it->second;
    }
    bool i8(const std::string& n, std::vector<uint64_t> shape, std::vector<int8_t>& out) {
        const Blob* b = get(n, "i8", shape, false);
        return b && (out = le_vector<int8_t>(b->data, b->e->length), true);
    }
    bool i16(const std::string& n, std::vector<uint64_t> shape, std::vector<int16_t>& out) {
        const Blob* b = get(n, "i16", shape, false);
        return b && (out = le_vector<int16_t>(b->data, b->e->length), true);
    }
    bool i32(const std::string& n, std::vector<uint64_t> shape, std::vector<int32_t>& out) {
        const Blob* b = get(n, "i32", shape, false);
        return b && (out = le_vector<int32_t>(b->data, b->e->length), true);
    }
    bool rescale(const std::string& n, uint64_t rows, RowRescale& out) {
        const Blob* b = get(n, "i32", {rows}, true);
        if (!b) return false;
        out.m = le_vector<int32_t>(b->data, b->e->length);
        out.s = (uint32_t)b->e->shift;
        return true;
    }
    bool scalar_rescale(const std::string& n, int32_t& m, uint32_t& s) {
        RowRescale r;
        if (!rescale(n, 1, r)) return false;
        m = r.m[0];
        s = r.s;
        return true;
    }
    bool linear(const std::string& n, uint64_t rows, uint64_t cols, Linear& l) {
        l.rows = (int)rows;
        l.cols = (int)cols;
        return i8(n + ".w", {rows, cols}, l.w) && i32(n + ".b", {rows}, l.b) && rescale(n + ".rescale", rows, l.rs);
    }
    // layernorm.rs:141 LayerNorm::with_beta_frac: the beta fraction fits the rescale shift.
    bool layernorm(const std::string& n, uint64_t d, uint32_t beta_frac, LayerNormP& ln) {
        if (!i16(n + ".g", {d}, ln.g) || !i32(n + ".b", {d}, ln.b) || !scalar_rescale(n + ".rescale", ln.m, ln.s))
            return false;
        if (beta_frac && !(beta_frac <= ln.s && ln.s <= 120 && ln.s - beta_frac <= 92))
            return fail(err_, "model.constants.ln_beta_frac: does not fit the shift of " + n);
        ln.beta_frac = beta_frac;
        return true;
    }
    // The GELU table of a block: 256 or 65,536 entries, i8 (or i16 in a version 2 file).
    bool gelu(const std::string& n, Block& B) {
        auto it = blobs_.find(n);
        if (it == blobs_.end()) return fail(err_, "missing tensor " + n);
        const std::vector<uint64_t>& sh = it->second.e->shape;
        if (sh.size() != 1 || (sh[0] != 256 && sh[0] != 65536))
            return fail(err_, "tensor " + n + ": a GELU table has 256 or 65536 entries");
        B.gelu_offset = sh[0] == 256 ? 128 : 32768;
        B.gelu_wide = it->second.e->dtype == "i16";
        return B.gelu_wide ? i16(n, sh, B.gelu16) : i8(n, sh, B.gelu8);
    }
    bool all_used() {
        for (auto& kv : blobs_)
            if (!kv.second.used) return fail(err_, "unexpected tensor " + kv.first + ": gpt2 does not use it");
        return true;
    }

  private:
    std::unordered_map<std::string, Blob>& blobs_;
    std::string& err_;
};

}  // namespace

bool Model::is_wide() const {
    if (ln_f_bits == 16 || ln_beta_frac > 0) return true;
    for (const Block& b : blocks)
        if (b.gelu_wide) return true;
    return false;
}

bool load_model(const uint8_t* f, size_t n, Model& M, std::string& err) {
    err.clear();
    // 1. Preamble.
    if (n < 16) return fail(err, "truncated: the preamble has 16 bytes");
    if (memcmp(f, "HSHLMDL\0", 8) != 0) return fail(err, "bad magic");
    uint32_t version, hlen;
    memcpy(&version, f + 8, 4);
    memcpy(&hlen, f + 12, 4);
    if (version != 1 && version != 2) return fail(err, "unsupported version " + std::to_string(version));
    if (hlen > n - 16) return fail(err, "truncated: the header runs past the end of the file");
    if (!utf8_ok(f + 16, hlen)) return fail(err, "the header is not UTF-8");
    // 2.-3. Header and model fields.
    Header h;
    if (!read_header((const char*)f + 16, (const char*)f + 16 + hlen, h, err)) return false;
    if (!check_fields(h, version, err)) return false;
    // 4. Sections: the vocabulary right after the header, then the merges, then the tensors.
    Sections sec(f, n, 16 + (uint64_t)hlen, err);
    const uint8_t* data;
    if (!sec.take(h.voff, h.vlen, "the vocabulary", &data) || !read_vocabulary(data, h.vlen, h.vocab, M, err))
        return false;
    M.merges.clear();
    if (h.has_merges && (!sec.take(h.moff, h.mlen, "the merges", &data) || !read_merges(data, h.mlen, M, err)))
        return false;
    std::unordered_map<std::string, Blob> blobs;
    for (const TensorEntry& t : h.tensors) {
        if (!good_name(t.name)) return fail(err, "tensors[].name: 1 to 128 characters from a-z 0-9 _ .");
        const size_t w = width_of(t.dtype);
        if (!w) return fail(err, "tensor " + t.name + ": unknown dtype");
        if (t.shape.empty() || t.shape.size() > 4) return fail(err, "tensor " + t.name + ": 1 to 4 dimensions");
        unsigned __int128 count = 1;
        for (uint64_t d : t.shape) {
            if (!d) return fail(err, "tensor " + t.name + ": a dimension is zero");
            count *= d;
            if (count > ((unsigned __int128)1 << 62)) return fail(err, "tensor " + t.name + ": too many elements");
        }
        if ((unsigned __int128)t.length != count * w) return fail(err, "tensor " + t.name + ": the length is not the shape's");
        if (t.has_shift && t.dtype != "i32") return fail(err, "tensor " + t.name + ": only i32 multipliers have a shift");
        if (!sec.take(t.offset, t.length, "tensor " + t.name, &data)) return false;
        if (!blobs.emplace(t.name, Blob{&t, data}).second) return fail(err, "tensor " + t.name + ": named two times");
    }
    if (!sec.at_end()) return false;
    // 5. The GPT-2 tensors.
    M.version = version;
    M.n_layer = (int)h.n_layer;
    M.n_head = (int)h.n_head;
    M.d_model = (int)h.d_model;
    M.d_ff = (int)h.d_ff;
    M.head_dim = (int)(h.d_model / h.n_head);
    M.vocab = (int)h.vocab;
    M.n_ctx = (int)h.n_ctx;
    M.eot = (uint32_t)h.eot;
    M.ln_k = (uint32_t)h.ln_k;
    M.ln_j = (uint32_t)h.ln_j;
    M.ln_eps = h.ln_eps;
    M.softmax_p = (uint32_t)h.softmax_p;
    M.ln_f_bits = h.has_lnf ? 16 : 8;
    M.ln_beta_frac = h.has_bf ? (uint32_t)h.beta_frac : 0;
    TensorSet ts(blobs, err);
    const uint64_t d = h.d_model, ff = h.d_ff, V = h.vocab, C = h.n_ctx;
    const uint32_t bf = M.ln_beta_frac;
    if (!ts.i8("wte", {V, d}, M.wte) || !ts.rescale("wte.rescale_embed", V, M.embed) ||
        !ts.rescale("wte.rescale_logits", V, M.logit) || !ts.i8("wpe", {C, d}, M.wpe) ||
        !ts.rescale("wpe.rescale", C, M.pos))
        return false;
    M.blocks.assign(M.n_layer, Block());
    for (int l = 0; l < M.n_layer; l++) {
        Block& B = M.blocks[l];
        const std::string p = "h." + std::to_string(l) + ".";
        if (!ts.layernorm(p + "ln_1", d, bf, B.ln_1) || !ts.linear(p + "attn.c_attn", 3 * d, d, B.c_attn) ||
            !ts.scalar_rescale(p + "attn.score.rescale", B.score_m, B.score_s) ||
            !ts.scalar_rescale(p + "attn.out.rescale", B.out_m, B.out_s) ||
            !ts.linear(p + "attn.c_proj", d, d, B.c_proj) || !ts.layernorm(p + "ln_2", d, bf, B.ln_2) ||
            !ts.linear(p + "mlp.c_fc", ff, d, B.c_fc) || !ts.gelu(p + "mlp.gelu", B) ||
            !ts.linear(p + "mlp.c_proj", d, ff, B.mlp_proj))
            return false;
    }
    if (!ts.layernorm("ln_f", d, bf, M.ln_f)) return false;
    if (!ts.i32("attn_exp", {}, M.attn_exp)) return false;
    if (!exp_table_ok(M.attn_exp)) return fail(err, "tensor attn_exp: entries >= 0, not increasing, the first >= 1");
    const Blob* lx = ts.get("logits_exp", "u64", {}, false);
    if (!lx) return false;
    M.logits_exp = le_vector<uint64_t>(lx->data, lx->e->length);
    bool lx_ok = exp_table_ok(M.logits_exp);
    for (uint64_t e : M.logits_exp) lx_ok = lx_ok && e <= (1ULL << 40);
    if (!lx_ok) return fail(err, "tensor logits_exp: entries <= 2^40, not increasing, the first >= 1");
    return ts.all_used();
}

}  // namespace hsm
