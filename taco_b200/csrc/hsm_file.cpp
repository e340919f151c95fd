// The .hsm reader and the GPT-2 model loader of the B200 backend (host side): it refuses every
// file that hardshell::gpt2::Model::load refuses. Each check follows the reference:
// - preamble, version and header length: crates/hardshell/src/hsm/reader.rs:357-380;
// - the JSON schema (deny_unknown_fields, integers only): hsm/header.rs:15-200;
// - check_config / check_version: hsm/reader.rs:270-320;
// - the section layout (align64, zero padding, exact end): hsm/reader.rs:382-440;
// - the vocabulary section: hsm/reader.rs:173-200; the merges: hsm/merges.rs:66-120;
// - the tensor table and the model dims: gpt2/model.rs:117-403.
#include "hsm_file.hpp"

#include <cstring>
#include <map>
#include <set>

namespace hsm {

namespace {

// ---- a small strict JSON parser (objects, arrays, strings, unsigned integers) ----

struct JVal {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    bool num_int = false;  // an integer literal without sign, fraction or exponent
    bool num_overflow = false;
    unsigned long long u = 0;
    std::string s;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
};

struct JParser {
    const char* p;
    const char* end;
    std::string err;

    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool fail(const char* m) {
        if (err.empty()) err = m;
        return false;
    }
    bool lit(const char* w) {
        size_t n = strlen(w);
        if ((size_t)(end - p) < n || memcmp(p, w, n) != 0) return false;
        p += n;
        return true;
    }
    static void put_utf8(std::string& o, uint32_t cp) {
        if (cp < 0x80) {
            o.push_back((char)cp);
        } else if (cp < 0x800) {
            o.push_back((char)(0xC0 | (cp >> 6)));
            o.push_back((char)(0x80 | (cp & 0x3F)));
        } else if (cp < 0x10000) {
            o.push_back((char)(0xE0 | (cp >> 12)));
            o.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            o.push_back((char)(0x80 | (cp & 0x3F)));
        } else {
            o.push_back((char)(0xF0 | (cp >> 18)));
            o.push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
            o.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            o.push_back((char)(0x80 | (cp & 0x3F)));
        }
    }
    bool hex4(uint32_t& v) {
        if (end - p < 4) return fail("truncated escape");
        v = 0;
        for (int i = 0; i < 4; i++) {
            char c = *p++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= c - '0';
            else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
            else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
            else return fail("bad escape");
        }
        return true;
    }
    bool str(std::string& o) {
        if (p >= end || *p != '"') return fail("expected a string");
        p++;
        while (true) {
            if (p >= end) return fail("unterminated string");
            unsigned char c = (unsigned char)*p++;
            if (c == '"') return true;
            if (c < 0x20) return fail("control character in string");
            if (c != '\\') {
                o.push_back((char)c);
                continue;
            }
            if (p >= end) return fail("truncated escape");
            char e = *p++;
            switch (e) {
                case '"': o.push_back('"'); break;
                case '\\': o.push_back('\\'); break;
                case '/': o.push_back('/'); break;
                case 'b': o.push_back('\b'); break;
                case 'f': o.push_back('\f'); break;
                case 'n': o.push_back('\n'); break;
                case 'r': o.push_back('\r'); break;
                case 't': o.push_back('\t'); break;
                case 'u': {
                    uint32_t v;
                    if (!hex4(v)) return false;
                    if (v >= 0xD800 && v < 0xDC00) {
                        uint32_t lo;
                        if (!lit("\\u") || !hex4(lo) || lo < 0xDC00 || lo >= 0xE000)
                            return fail("bad surrogate pair");
                        v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (v >= 0xDC00 && v < 0xE000) {
                        return fail("lone surrogate");
                    }
                    put_utf8(o, v);
                    break;
                }
                default: return fail("bad escape");
            }
        }
    }
    bool num(JVal& v) {
        v.kind = JVal::Num;
        bool neg = false;
        if (*p == '-') {
            neg = true;
            p++;
        }
        if (p >= end || *p < '0' || *p > '9') return fail("bad number");
        const char* start = p;
        if (*p == '0' && p + 1 < end && p[1] >= '0' && p[1] <= '9') return fail("leading zero");
        unsigned long long u = 0;
        bool ovf = false;
        while (p < end && *p >= '0' && *p <= '9') {
            unsigned d = (unsigned)(*p - '0');
            if (u > (~0ULL - d) / 10) ovf = true;
            u = u * 10 + d;
            p++;
        }
        bool frac = false;
        if (p < end && *p == '.') {
            frac = true;
            p++;
            if (p >= end || *p < '0' || *p > '9') return fail("bad number");
            while (p < end && *p >= '0' && *p <= '9') p++;
        }
        if (p < end && (*p == 'e' || *p == 'E')) {
            frac = true;
            p++;
            if (p < end && (*p == '+' || *p == '-')) p++;
            if (p >= end || *p < '0' || *p > '9') return fail("bad number");
            while (p < end && *p >= '0' && *p <= '9') p++;
        }
        (void)start;
        v.num_int = !neg && !frac;
        v.num_overflow = ovf;
        v.u = u;
        return true;
    }
    bool value(JVal& v, int depth) {
        if (depth > 64) return fail("too deep");
        ws();
        if (p >= end) return fail("unexpected end");
        char c = *p;
        if (c == '{') {
            p++;
            v.kind = JVal::Obj;
            ws();
            if (p < end && *p == '}') {
                p++;
                return true;
            }
            while (true) {
                ws();
                std::string k;
                if (!str(k)) return false;
                for (auto& kv : v.obj)
                    if (kv.first == k) return fail("duplicate field");
                ws();
                if (p >= end || *p != ':') return fail("expected ':'");
                p++;
                JVal child;
                if (!value(child, depth + 1)) return false;
                v.obj.emplace_back(k, std::move(child));
                ws();
                if (p < end && *p == ',') {
                    p++;
                    continue;
                }
                if (p < end && *p == '}') {
                    p++;
                    return true;
                }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            p++;
            v.kind = JVal::Arr;
            ws();
            if (p < end && *p == ']') {
                p++;
                return true;
            }
            while (true) {
                JVal child;
                if (!value(child, depth + 1)) return false;
                v.arr.push_back(std::move(child));
                ws();
                if (p < end && *p == ',') {
                    p++;
                    continue;
                }
                if (p < end && *p == ']') {
                    p++;
                    return true;
                }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = JVal::Str;
            return str(v.s);
        }
        if (c == 't') {
            if (!lit("true")) return fail("bad literal");
            v.kind = JVal::Bool;
            v.b = true;
            return true;
        }
        if (c == 'f') {
            if (!lit("false")) return fail("bad literal");
            v.kind = JVal::Bool;
            return true;
        }
        if (c == 'n') {
            if (!lit("null")) return fail("bad literal");
            v.kind = JVal::Null;
            return true;
        }
        return num(v);
    }
};

// Reads the fields of an object against a fixed schema: every field known, each at most once.
struct Fields {
    const JVal* obj;
    std::string* err;
    std::string where;
    std::set<std::string> seen = {};

    const JVal* get(const char* name, bool required) {
        for (auto& kv : obj->obj) {
            if (kv.first == name) {
                seen.insert(name);
                return &kv.second;
            }
        }
        if (required && err->empty()) *err = "header: missing field " + where + name;
        return nullptr;
    }
    bool uint(const char* name, unsigned long long max, unsigned long long& out, bool required = true) {
        const JVal* v = get(name, required);
        if (!v) return !required;
        if (v->kind != JVal::Num || !v->num_int || v->num_overflow || v->u > max) {
            if (err->empty()) *err = "header: field " + where + name + " is not a valid integer";
            return false;
        }
        out = v->u;
        return true;
    }
    bool string(const char* name, std::string& out) {
        const JVal* v = get(name, true);
        if (!v) return false;
        if (v->kind != JVal::Str) {
            if (err->empty()) *err = "header: field " + where + name + " is not a string";
            return false;
        }
        out = v->s;
        return true;
    }
    bool no_unknown() {
        for (auto& kv : obj->obj) {
            if (!seen.count(kv.first)) {
                if (err->empty()) *err = "header: unknown field " + where + kv.first;
                return false;
            }
        }
        return true;
    }
};

uint64_t align64(uint64_t x) { return (x + 63) & ~(uint64_t)63; }

bool valid_name(const std::string& n) {
    if (n.empty() || n.size() > 128) return false;
    for (unsigned char c : n)
        if (!((c >= 'a' && c <= 'z') || (c >= '0' && c <= '9') || c == '_' || c == '.')) return false;
    return true;
}

struct Entry {
    std::string name, dtype;
    std::vector<uint64_t> shape;
    unsigned long long offset = 0, length = 0;
    bool has_shift = false;
    uint32_t shift = 0;
};

struct Raw {
    std::string dtype;
    std::vector<uint64_t> shape;
    const uint8_t* data = nullptr;
    size_t length = 0;
    bool has_shift = false;
    uint32_t shift = 0;
    bool taken = false;
};

size_t dtype_size(const std::string& d) {
    if (d == "i8") return 1;
    if (d == "i16") return 2;
    if (d == "i32") return 4;
    if (d == "u64") return 8;
    return 0;
}

template <typename T>
std::vector<T> decode_le(const uint8_t* p, size_t n) {
    std::vector<T> v(n);
    memcpy(v.data(), p, n * sizeof(T));  // little-endian host (x86-64)
    return v;
}

struct Loader {
    std::map<std::string, Raw>& t;
    std::string& err;

    Raw* take(const std::string& name, const std::vector<uint64_t>& dims, bool shift) {
        auto it = t.find(name);
        if (it == t.end() || it->second.taken) {
            if (err.empty()) err = "missing tensor " + name;
            return nullptr;
        }
        Raw& r = it->second;
        if (r.shape != dims) {
            if (err.empty()) err = "tensor " + name + ": the shape is not the shape that the model needs";
            return nullptr;
        }
        if (shift && !r.has_shift) {
            if (err.empty()) err = "tensor " + name + ": a rescale tensor needs a shift";
            return nullptr;
        }
        if (!shift && r.has_shift) {
            if (err.empty()) err = "tensor " + name + ": only a rescale tensor has a shift";
            return nullptr;
        }
        r.taken = true;
        return &r;
    }
    bool typed(Raw* r, const char* dt, const std::string& name) {
        if (!r) return false;
        if (r->dtype != dt) {
            if (err.empty()) err = "tensor " + name + ": the dtype is not the dtype that the model needs";
            return false;
        }
        return true;
    }
    bool i8(const std::string& name, std::vector<uint64_t> dims, std::vector<int8_t>& out) {
        Raw* r = take(name, dims, false);
        if (!typed(r, "i8", name)) return false;
        out = decode_le<int8_t>(r->data, r->length);
        return true;
    }
    bool i16(const std::string& name, std::vector<uint64_t> dims, std::vector<int16_t>& out) {
        Raw* r = take(name, dims, false);
        if (!typed(r, "i16", name)) return false;
        out = decode_le<int16_t>(r->data, r->length / 2);
        return true;
    }
    bool i32(const std::string& name, std::vector<uint64_t> dims, std::vector<int32_t>& out) {
        Raw* r = take(name, dims, false);
        if (!typed(r, "i32", name)) return false;
        out = decode_le<int32_t>(r->data, r->length / 4);
        return true;
    }
    bool rows_rescale(const std::string& name, uint64_t len, RowRescale& out) {
        Raw* r = take(name, {len}, true);
        if (!typed(r, "i32", name)) return false;
        out.m = decode_le<int32_t>(r->data, r->length / 4);
        out.s = r->shift;
        return true;
    }
    bool rescale1(const std::string& name, int32_t& m, uint32_t& s) {
        RowRescale rr;
        if (!rows_rescale(name, 1, rr)) return false;
        m = rr.m[0];
        s = rr.s;
        return true;
    }
    bool linear(const std::string& p, int rows, int cols, Linear& l) {
        l.rows = rows;
        l.cols = cols;
        return i8(p + ".w", {(uint64_t)rows, (uint64_t)cols}, l.w) && i32(p + ".b", {(uint64_t)rows}, l.b) &&
               rows_rescale(p + ".rescale", rows, l.rs);
    }
    // layernorm.rs:141 LayerNorm::with_beta_frac checks.
    bool layernorm(const std::string& p, int d, uint32_t beta_frac, LayerNormP& ln) {
        if (!i16(p + ".g", {(uint64_t)d}, ln.g) || !i32(p + ".b", {(uint64_t)d}, ln.b) ||
            !rescale1(p + ".rescale", ln.m, ln.s))
            return false;
        if (beta_frac > 0) {
            bool ok = beta_frac <= 16 && beta_frac <= ln.s && ln.s <= 120 && ln.s - beta_frac <= 92;
            if (!ok) {
                if (err.empty()) err = "model.constants.ln_beta_frac: out of range for " + p;
                return false;
            }
        }
        ln.beta_frac = beta_frac;
        return true;
    }
};

// softmax.rs:60 is_valid_exp_table: not empty, >= min, not increasing, first >= 1.
template <typename T>
bool valid_exp_table(const std::vector<T>& e) {
    if (e.empty() || e[0] < (T)1) return false;
    for (size_t i = 0; i < e.size(); i++) {
        if (e[i] < (T)0) return false;
        if (i > 0 && e[i] > e[i - 1]) return false;
    }
    return true;
}

}  // namespace

bool Model::is_wide() const {
    if (ln_f_bits == 16 || ln_beta_frac > 0) return true;
    for (auto& b : blocks)
        if (b.gelu_wide) return true;
    return false;
}

bool load_model(const uint8_t* bytes, size_t len, Model& M, std::string& err) {
    err.clear();
    if (len < 16) {
        err = "truncated: the preamble needs 16 bytes";
        return false;
    }
    if (memcmp(bytes, "HSHLMDL\0", 8) != 0) {
        err = "bad magic";
        return false;
    }
    uint32_t version, header_len;
    memcpy(&version, bytes + 8, 4);
    memcpy(&header_len, bytes + 12, 4);
    if (version != 1 && version != 2) {
        err = "unsupported version";
        return false;
    }
    if ((uint64_t)16 + header_len > len) {
        err = "truncated header";
        return false;
    }
    JParser jp{(const char*)bytes + 16, (const char*)bytes + 16 + header_len, {}};
    JVal root;
    if (!jp.value(root, 0)) {
        err = "header JSON: " + jp.err;
        return false;
    }
    jp.ws();
    if (jp.p != jp.end) {
        err = "header JSON: trailing characters";
        return false;
    }
    if (root.kind != JVal::Obj) {
        err = "header JSON: not an object";
        return false;
    }
    Fields top{&root, &err, ""};
    const JVal* model = top.get("model", true);
    const JVal* vocab = top.get("vocabulary", true);
    const JVal* merges = top.get("merges", false);
    const JVal* tensors = top.get("tensors", true);
    if (!err.empty() || !top.no_unknown()) return false;
    if (model->kind != JVal::Obj || vocab->kind != JVal::Obj || tensors->kind != JVal::Arr ||
        (merges && merges->kind != JVal::Obj)) {
        err = "header: wrong field types";
        return false;
    }
    Fields mf{model, &err, "model."};
    std::string arch;
    unsigned long long n_layer, n_head, d_model, d_ff, vocab_size, n_ctx, eot;
    if (!mf.string("architecture", arch) || !mf.uint("n_layer", 0xFFFFFFFFull, n_layer) ||
        !mf.uint("n_head", 0xFFFFFFFFull, n_head) || !mf.uint("d_model", 0xFFFFFFFFull, d_model) ||
        !mf.uint("d_ff", 0xFFFFFFFFull, d_ff) || !mf.uint("vocab_size", 0xFFFFFFFFull, vocab_size) ||
        !mf.uint("n_ctx", 0xFFFFFFFFull, n_ctx) || !mf.uint("eot_token", 0xFFFFFFFFull, eot))
        return false;
    const JVal* consts = mf.get("constants", true);
    if (!consts || !mf.no_unknown()) return false;
    if (consts->kind != JVal::Obj) {
        err = "header: constants is not an object";
        return false;
    }
    Fields cf{consts, &err, "model.constants."};
    unsigned long long ln_k, ln_j, ln_eps, softmax_p, ln_f_bits = 0, ln_beta_frac = 0;
    if (!cf.uint("ln_k", 255, ln_k) || !cf.uint("ln_j", 255, ln_j) || !cf.uint("ln_eps", ~0ULL, ln_eps) ||
        !cf.uint("softmax_p", 255, softmax_p))
        return false;
    bool has_lnf = cf.get("ln_f_bits", false) != nullptr;
    bool has_bf = cf.get("ln_beta_frac", false) != nullptr;
    if (has_lnf && !cf.uint("ln_f_bits", 255, ln_f_bits, true)) return false;
    if (has_bf && !cf.uint("ln_beta_frac", 255, ln_beta_frac, true)) return false;
    if (!cf.no_unknown()) return false;
    Fields vf{vocab, &err, "vocabulary."};
    unsigned long long voff, vlen, moff = 0, mlen = 0;
    if (!vf.uint("offset", ~0ULL, voff) || !vf.uint("length", ~0ULL, vlen) || !vf.no_unknown()) return false;
    if (merges) {
        Fields gf{merges, &err, "merges."};
        if (!gf.uint("offset", ~0ULL, moff) || !gf.uint("length", ~0ULL, mlen) || !gf.no_unknown()) return false;
    }
    std::vector<Entry> entries;
    for (auto& tv : tensors->arr) {
        if (tv.kind != JVal::Obj) {
            err = "header: a tensor entry is not an object";
            return false;
        }
        Fields tf{&tv, &err, "tensors[]."};
        Entry e;
        const JVal* shape;
        unsigned long long shift = 0;
        if (!tf.string("name", e.name) || !tf.string("dtype", e.dtype)) return false;
        shape = tf.get("shape", true);
        if (!shape) return false;
        if (!tf.uint("offset", ~0ULL, e.offset) || !tf.uint("length", ~0ULL, e.length)) return false;
        e.has_shift = tf.get("shift", false) != nullptr;
        if (e.has_shift) {
            if (!tf.uint("shift", 255, shift, true)) return false;
            e.shift = (uint32_t)shift;
        }
        if (!tf.no_unknown()) return false;
        if (shape->kind != JVal::Arr) {
            err = "header: shape is not an array";
            return false;
        }
        for (auto& d : shape->arr) {
            if (d.kind != JVal::Num || !d.num_int || d.num_overflow) {
                err = "header: a shape dimension is not an integer";
                return false;
            }
            e.shape.push_back(d.u);
        }
        entries.push_back(std::move(e));
    }
    // check_config (reader.rs)
    if (!valid_name(arch)) {
        err = "model.architecture: must have 1 to 128 characters from a-z 0-9 _ .";
        return false;
    }
    if (vocab_size == 0 || vocab_size > (1u << 20)) {
        err = "model.vocab_size: must be in 1..=2^20";
        return false;
    }
    if (eot >= vocab_size) {
        err = "model.eot_token: must be less than vocab_size";
        return false;
    }
    if (ln_k > 48 || ln_j > 16 || ln_eps == 0 || ln_eps > (1ULL << 62)) {
        err = "model.constants: LayerNorm constants out of range";
        return false;
    }
    if (softmax_p > 30) {
        err = "model.constants.softmax_p: must be at most 30";
        return false;
    }
    // check_version
    if (has_lnf && ln_f_bits != 16) {
        err = "model.constants.ln_f_bits: must be 16";
        return false;
    }
    if (has_bf && (ln_beta_frac == 0 || ln_beta_frac > 16)) {
        err = "model.constants.ln_beta_frac: must be in 1..=16";
        return false;
    }
    bool wide_gelu = false;
    for (auto& e : entries) {
        size_t n = e.name.size();
        if (n >= 9 && e.name.compare(n - 9, 9, ".mlp.gelu") == 0 && e.dtype == "i16") wide_gelu = true;
    }
    uint32_t required = (has_lnf || has_bf || wide_gelu) ? 2 : 1;
    if (required != version) {
        err = "version: a file is version 2 if and only if it has a version 2 constant or an i16 GELU table";
        return false;
    }
    // Layout
    uint64_t header_end = 16 + (uint64_t)header_len;
    uint64_t vocab_offset = align64(header_end);
    if (voff != vocab_offset) {
        err = "layout: the vocabulary offset is not align64(16 + header_len)";
        return false;
    }
    auto check_pad = [&](uint64_t from, uint64_t to) -> bool {
        if (to > len) to = len;
        for (uint64_t i = from; i < to; i++)
            if (bytes[i] != 0) {
                err = "non-zero padding";
                return false;
            }
        return true;
    };
    if (vocab_offset > len) {
        err = "truncated";
        return false;
    }
    if (!check_pad(header_end, vocab_offset)) return false;
    if (vlen > len - vocab_offset) {
        err = "truncated vocabulary";
        return false;
    }
    // Vocabulary
    {
        const uint8_t* s = bytes + vocab_offset;
        uint64_t pos = 0;
        M.vocab_bytes.clear();
        M.vocab_ends.clear();
        for (uint64_t t = 0; t < vocab_size; t++) {
            if (pos + 2 > vlen) {
                err = "vocabulary: the length is outside the section";
                return false;
            }
            uint16_t l = (uint16_t)(s[pos] | (s[pos + 1] << 8));
            pos += 2;
            if (pos + l > vlen) {
                err = "vocabulary: the bytes are outside the section";
                return false;
            }
            M.vocab_bytes.insert(M.vocab_bytes.end(), s + pos, s + pos + l);
            M.vocab_ends.push_back(M.vocab_bytes.size());
            pos += l;
        }
        if (pos != vlen) {
            err = "vocabulary: the section has extra bytes";
            return false;
        }
    }
    uint64_t cursor = vocab_offset + vlen;
    if (merges) {
        uint64_t off = align64(cursor);
        if (moff != off) {
            err = "layout: the merges offset is not align64 of the vocabulary end";
            return false;
        }
        if (!check_pad(cursor, off)) return false;
        if (off > len || mlen > len - off) {
            err = "truncated merges";
            return false;
        }
        if (mlen == 0 || mlen % 8 != 0) {
            err = "merges.length: must be a multiple of 8 and at least 8";
            return false;
        }
        // merges.rs:66 parse: ids in range, parts not empty, no duplicate pair, the joined
        // bytes are the bytes of exactly one token.
        std::map<std::string, long long> by_bytes;
        for (uint64_t i = 0; i < vocab_size; i++) {
            size_t a = i ? M.vocab_ends[i - 1] : 0, b = M.vocab_ends[i];
            std::string k((const char*)M.vocab_bytes.data() + a, b - a);
            auto it = by_bytes.find(k);
            if (it == by_bytes.end()) by_bytes[k] = (long long)i;
            else it->second = -1;
        }
        std::set<std::pair<uint32_t, uint32_t>> seen;
        const uint8_t* s = bytes + off;
        for (uint64_t r = 0; r < mlen / 8; r++) {
            uint32_t l, rr;
            memcpy(&l, s + 8 * r, 4);
            memcpy(&rr, s + 8 * r + 4, 4);
            if (l >= vocab_size || rr >= vocab_size) {
                err = "merges: an id is not in the vocabulary";
                return false;
            }
            size_t la = l ? M.vocab_ends[l - 1] : 0, lb = M.vocab_ends[l];
            size_t ra = rr ? M.vocab_ends[rr - 1] : 0, rb = M.vocab_ends[rr];
            if (la == lb || ra == rb) {
                err = "merges: a part has no bytes";
                return false;
            }
            if (!seen.insert({l, rr}).second) {
                err = "merges: a pair occurs two times";
                return false;
            }
            std::string joined((const char*)M.vocab_bytes.data() + la, lb - la);
            joined.append((const char*)M.vocab_bytes.data() + ra, rb - ra);
            auto it = by_bytes.find(joined);
            if (it == by_bytes.end() || it->second < 0) {
                err = "merges: the joined bytes are not the bytes of exactly one token";
                return false;
            }
            M.merges.push_back({l, rr});
        }
        cursor = off + mlen;
    }
    std::map<std::string, Raw> raw;
    for (auto& e : entries) {
        if (!valid_name(e.name)) {
            err = "tensors[].name: must have 1 to 128 characters from a-z 0-9 _ .";
            return false;
        }
        if (raw.count(e.name)) {
            err = "tensor " + e.name + ": the name occurs two times";
            return false;
        }
        size_t ds = dtype_size(e.dtype);
        if (!ds) {
            err = "tensor " + e.name + ": unknown dtype";
            return false;
        }
        if (e.shape.empty() || e.shape.size() > 4) {
            err = "tensor " + e.name + ": a shape has 1 to 4 dimensions";
            return false;
        }
        unsigned __int128 numel = 1;
        for (auto d : e.shape) {
            if (d == 0) {
                err = "tensor " + e.name + ": a dimension is zero";
                return false;
            }
            numel *= d;
            if (numel > ((unsigned __int128)1 << 62)) {
                err = "tensor " + e.name + ": the element count overflows";
                return false;
            }
        }
        if ((unsigned __int128)e.length != numel * ds) {
            err = "tensor " + e.name + ": length is not product(shape) * dtype size";
            return false;
        }
        if (e.has_shift && e.dtype != "i32") {
            err = "tensor " + e.name + ": only an i32 tensor of rescale multipliers has a shift";
            return false;
        }
        uint64_t off = align64(cursor);
        if (e.offset != off) {
            err = "layout: tensor " + e.name + ": the offset is not align64 of the end of the section before";
            return false;
        }
        if (!check_pad(cursor, off)) return false;
        if (off > len || e.length > len - off) {
            err = "truncated tensor " + e.name;
            return false;
        }
        Raw r;
        r.dtype = e.dtype;
        r.shape = e.shape;
        r.data = bytes + off;
        r.length = e.length;
        r.has_shift = e.has_shift;
        r.shift = e.shift;
        raw[e.name] = r;
        cursor = off + e.length;
    }
    if (cursor != len) {
        err = "layout: the file does not end at the end of the last section";
        return false;
    }
    // gpt2/model.rs:117 check_dims
    if (arch != "gpt2") {
        err = "model.architecture: this loader reads only \"gpt2\"";
        return false;
    }
    if (n_layer == 0 || n_layer > 1024) {
        err = "model.n_layer: must be in 1..=1024";
        return false;
    }
    if (d_model == 0 || d_model > 65536) {
        err = "model.d_model: must be in 1..=65536";
        return false;
    }
    if (d_ff == 0 || d_ff > 65536) {
        err = "model.d_ff: must be in 1..=65536";
        return false;
    }
    if (n_head == 0 || d_model % n_head != 0) {
        err = "model.n_head: must be at least 1 and divide d_model";
        return false;
    }
    if (n_ctx < 2 || n_ctx > 65536) {
        err = "model.n_ctx: must be in 2..=65536";
        return false;
    }
    M.version = version;
    M.n_layer = (int)n_layer;
    M.n_head = (int)n_head;
    M.d_model = (int)d_model;
    M.d_ff = (int)d_ff;
    M.head_dim = (int)(d_model / n_head);
    M.vocab = (int)vocab_size;
    M.n_ctx = (int)n_ctx;
    M.eot = (uint32_t)eot;
    M.ln_k = (uint32_t)ln_k;
    M.ln_j = (uint32_t)ln_j;
    M.ln_eps = ln_eps;
    M.softmax_p = (uint32_t)softmax_p;
    M.ln_f_bits = has_lnf ? 16 : 8;
    M.ln_beta_frac = has_bf ? (uint32_t)ln_beta_frac : 0;
    Loader ld{raw, err};
    int d = M.d_model, f = M.d_ff, V = M.vocab, C = M.n_ctx;
    if (!ld.i8("wte", {(uint64_t)V, (uint64_t)d}, M.wte) || !ld.rows_rescale("wte.rescale_embed", V, M.embed) ||
        !ld.rows_rescale("wte.rescale_logits", V, M.logit) || !ld.i8("wpe", {(uint64_t)C, (uint64_t)d}, M.wpe) ||
        !ld.rows_rescale("wpe.rescale", C, M.pos))
        return false;
    M.blocks.resize(M.n_layer);
    for (int l = 0; l < M.n_layer; l++) {
        Block& B = M.blocks[l];
        std::string p = "h." + std::to_string(l);
        if (!ld.layernorm(p + ".ln_1", d, M.ln_beta_frac, B.ln_1) ||
            !ld.linear(p + ".attn.c_attn", 3 * d, d, B.c_attn) ||
            !ld.rescale1(p + ".attn.score.rescale", B.score_m, B.score_s) ||
            !ld.rescale1(p + ".attn.out.rescale", B.out_m, B.out_s) ||
            !ld.linear(p + ".attn.c_proj", d, d, B.c_proj) || !ld.layernorm(p + ".ln_2", d, M.ln_beta_frac, B.ln_2) ||
            !ld.linear(p + ".mlp.c_fc", f, d, B.c_fc))
            return false;
        std::string gn = p + ".mlp.gelu";
        auto it = raw.find(gn);
        if (it == raw.end()) {
            err = "missing tensor " + gn;
            return false;
        }
        uint64_t glen = it->second.shape.empty() ? 0 : it->second.shape[0];
        if (glen != 256 && glen != 65536) {
            err = "tensor " + gn + ": a GELU table has 256 or 65536 entries";
            return false;
        }
        if (it->second.dtype == "i16") {
            B.gelu_wide = true;
            if (!ld.i16(gn, {glen}, B.gelu16)) return false;
        } else {
            if (!ld.i8(gn, {glen}, B.gelu8)) return false;
        }
        B.gelu_offset = glen == 256 ? 128 : 32768;
        if (!ld.linear(p + ".mlp.c_proj", d, f, B.mlp_proj)) return false;
    }
    if (!ld.layernorm("ln_f", d, M.ln_beta_frac, M.ln_f)) return false;
    {
        auto it = raw.find("attn_exp");
        if (it == raw.end()) {
            err = "missing tensor attn_exp";
            return false;
        }
        if (it->second.shape.size() != 1) {
            err = "tensor attn_exp: a table has one dimension";
            return false;
        }
        if (!ld.i32("attn_exp", it->second.shape, M.attn_exp)) return false;
        if (!valid_exp_table(M.attn_exp)) {
            err = "tensor attn_exp: entries must be >= 0, not increasing, and the first entry >= 1";
            return false;
        }
    }
    {
        auto it = raw.find("logits_exp");
        if (it == raw.end()) {
            err = "missing tensor logits_exp";
            return false;
        }
        if (it->second.shape.size() != 1) {
            err = "tensor logits_exp: a table has one dimension";
            return false;
        }
        Raw* r = ld.take("logits_exp", it->second.shape, false);
        if (!ld.typed(r, "u64", "logits_exp")) return false;
        M.logits_exp = decode_le<uint64_t>(r->data, r->length / 8);
        bool ok = valid_exp_table(M.logits_exp);
        for (auto e : M.logits_exp)
            if (e > (1ULL << 40)) ok = false;
        if (!ok) {
            err = "tensor logits_exp: entries must be <= 2^40, not increasing, and the first entry >= 1";
            return false;
        }
    }
    for (auto& kv : raw) {
        if (!kv.second.taken) {
            err = "unexpected tensor " + kv.first + ": the gpt2 model does not use this tensor";
            return false;
        }
    }
    return true;
}

}  // namespace hsm
