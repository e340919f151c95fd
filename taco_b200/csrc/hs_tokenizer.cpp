// The tokenizer of the fold: GPT-2 byte-level BPE over the vocabulary and the merges of a .hsm
// model (crates/taco/src/tokenizer/mod.rs Tokenizer, pretokenize.rs Pieces, bpe.rs merge_into).
// Host code only; it needs no GPU.
//
// Any byte string tokenizes: the input divides into maximal runs of well-formed UTF-8 and the
// single bytes outside them (mod.rs:1-12). A run goes through the GPT-2 pre-tokenizer, the pattern
//   's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+
// (pretokenize.rs), and each piece through the merges: the pair of lowest rank first, all of its
// places from the left (bpe.rs). A byte outside a run is its single-byte token. The bytes of the
// tokens join to the input, for every input.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <queue>
#include <string>
#include <unordered_map>
#include <vector>

#include "hardshell_b200.h"
#include "hs_host.hpp"
#include "hsm_file.hpp"

namespace {

struct CodeRange {
    uint32_t lo, hi;
};
#include "hs_unicode.inc"

template <size_t N>
bool in_table(const CodeRange (&t)[N], uint32_t c) {
    size_t lo = 0, hi = N;
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (t[mid].hi < c) lo = mid + 1;
        else if (t[mid].lo > c) hi = mid;
        else return true;
    }
    return false;
}

enum CharClass : uint8_t { LETTER, NUMBER, SPACE, OTHER };

// The class of a code point: \p{L}, \p{N}, White_Space, or none of them.
CharClass class_of(uint32_t c) {
    if (c < 128) {
        if ((c | 32u) - 'a' < 26u) return LETTER;
        if (c - '0' < 10u) return NUMBER;
        if (c == ' ' || (c >= 9 && c <= 13)) return SPACE;
        return OTHER;
    }
    if (in_table(kLetter, c)) return LETTER;
    if (in_table(kNumber, c)) return NUMBER;
    if (in_table(kWhiteSpace, c)) return SPACE;
    return OTHER;
}

// The length of the well-formed UTF-8 character at p (Unicode table 3-7), or 0 if the bytes at p
// do not start one. A byte that does not start one is outside every run: a byte of an ill-formed
// sequence never starts a well-formed character either, so deciding byte by byte gives the runs
// of Rust's Utf8Chunks.
int utf8_char(const uint8_t* p, const uint8_t* end, uint32_t* cp) {
    const uint8_t b0 = p[0];
    if (b0 < 0x80) {
        *cp = b0;
        return 1;
    }
    int n;
    uint32_t c;
    uint8_t lo = 0x80, hi = 0xBF;
    if (b0 >= 0xC2 && b0 <= 0xDF) {
        n = 2;
        c = b0 & 0x1Fu;
    } else if (b0 >= 0xE0 && b0 <= 0xEF) {
        n = 3;
        c = b0 & 0x0Fu;
        if (b0 == 0xE0) lo = 0xA0;
        if (b0 == 0xED) hi = 0x9F;
    } else if (b0 >= 0xF0 && b0 <= 0xF4) {
        n = 4;
        c = b0 & 0x07u;
        if (b0 == 0xF0) lo = 0x90;
        if (b0 == 0xF4) hi = 0x8F;
    } else {
        return 0;
    }
    if (end - p < n) return 0;
    for (int i = 1; i < n; i++) {
        const uint8_t b = p[i];
        if (b < (i == 1 ? lo : 0x80) || b > (i == 1 ? hi : 0xBF)) return 0;
        c = (c << 6) | (b & 0x3Fu);
    }
    *cp = c;
    return n;
}

struct Char {
    size_t off;  // byte offset of the character in the input
    uint32_t cp;
    CharClass cls;
};

// The end (a character index) of the piece that starts at character i of a run.
size_t piece_end(const std::vector<Char>& ch, size_t i) {
    const size_t n = ch.size();
    if (ch[i].cp == '\'' && i + 1 < n) {
        const uint32_t a = ch[i + 1].cp, b = i + 2 < n ? ch[i + 2].cp : 0;
        if (a == 's' || a == 't' || a == 'm' || a == 'd') return i + 2;
        if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return i + 3;
    }
    size_t start = i;
    CharClass run = ch[i].cls;
    if (run == SPACE) {
        if (!(ch[i].cp == ' ' && i + 1 < n && ch[i + 1].cls != SPACE)) {
            // \s+(?!\S)|\s+: the white space up to the last one before a non-space character,
            // which starts the next piece (unless the run is a single character); all of it at
            // the end of the run.
            size_t k = i;
            while (k < n && ch[k].cls == SPACE) k++;
            if (k == n) return n;
            return k - i >= 2 ? k - 1 : k;
        }
        start = i + 1;  // " ?X+": one space, then a run of the next class
        run = ch[i + 1].cls;
    }
    size_t k = start;
    while (k < n && ch[k].cls == run) k++;
    return k;
}

struct Merge {
    uint32_t rank, merged;
};

uint64_t pair_key(uint32_t a, uint32_t b) { return (uint64_t)a << 32 | b; }

}  // namespace

struct hs_tokenizer {
    uint32_t byte_tokens[256];
    std::unordered_map<uint64_t, Merge> merges;
    uint32_t vocab = 0, eot = 0, n_ctx = 0;
    std::vector<uint8_t> bytes;  // the bytes of every token, joined
    std::vector<size_t> ends;    // the end of token i in `bytes`

    // The merges of one piece (bpe.rs merge_into): the pairs of the lowest rank left, all of them
    // in the order of their places, then again; a place whose pair changed is skipped.
    void merge_piece(const uint32_t* sym0, size_t n, std::vector<uint32_t>& out) const {
        if (n < 2) {
            out.insert(out.end(), sym0, sym0 + n);
            return;
        }
        constexpr size_t NONE = ~(size_t)0;
        std::vector<uint32_t> sym(sym0, sym0 + n);
        std::vector<size_t> next(n), prev(n);
        std::vector<char> alive(n, 1);
        for (size_t i = 0; i < n; i++) {
            next[i] = i + 1 < n ? i + 1 : NONE;
            prev[i] = i ? i - 1 : NONE;
        }
        using Entry = std::pair<uint32_t, size_t>;  // (rank, place)
        std::priority_queue<Entry, std::vector<Entry>, std::greater<Entry>> heap;
        auto merge_at = [&](size_t i) -> const Merge* {
            if (i == NONE || next[i] == NONE) return nullptr;
            auto it = merges.find(pair_key(sym[i], sym[next[i]]));
            return it == merges.end() ? nullptr : &it->second;
        };
        for (size_t i = 0; i + 1 < n; i++)
            if (const Merge* m = merge_at(i)) heap.push({m->rank, i});
        std::vector<size_t> batch;
        while (!heap.empty()) {
            const uint32_t rank = heap.top().first;
            batch.clear();
            while (!heap.empty() && heap.top().first == rank) {
                batch.push_back(heap.top().second);
                heap.pop();
            }
            std::sort(batch.begin(), batch.end());
            batch.erase(std::unique(batch.begin(), batch.end()), batch.end());
            for (size_t i : batch) {
                if (!alive[i]) continue;
                const Merge* m = merge_at(i);
                if (!m || m->rank != rank) continue;
                const size_t j = next[i], after = next[j];
                sym[i] = m->merged;
                alive[j] = 0;
                next[i] = after;
                if (after != NONE) prev[after] = i;
                for (size_t k : {prev[i], i})
                    if (const Merge* mk = merge_at(k)) heap.push({mk->rank, k});
            }
        }
        for (size_t i = 0; i != NONE; i = next[i]) out.push_back(sym[i]);
    }

    // Pieces of `data` as (start, end) byte offsets: the runs' pieces and the single bytes.
    template <typename F>
    void pieces(const uint8_t* data, size_t len, F&& on_piece, std::vector<Char>& ch) const {
        size_t i = 0;
        while (i < len) {
            ch.clear();
            uint32_t cp;
            int nb;
            while (i < len && (nb = utf8_char(data + i, data + len, &cp)) > 0) {
                ch.push_back({i, cp, class_of(cp)});
                i += (size_t)nb;
            }
            const size_t run_end = i;
            for (size_t c = 0; c < ch.size();) {
                const size_t e = piece_end(ch, c);
                on_piece(ch[c].off, e < ch.size() ? ch[e].off : run_end, true);
                c = e;
            }
            if (i < len) {
                on_piece(i, i + 1, false);  // a byte outside every run
                i++;
            }
        }
    }

    void encode(const uint8_t* data, size_t len, std::vector<uint32_t>& out) const {
        std::vector<Char> ch;
        std::vector<uint32_t> sym;
        pieces(
            data, len,
            [&](size_t a, size_t b, bool) {
                sym.clear();
                for (size_t k = a; k < b; k++) sym.push_back(byte_tokens[data[k]]);
                merge_piece(sym.data(), sym.size(), out);
            },
            ch);
    }
};

namespace {

// Tokenizer::new (mod.rs:80-130): every byte has exactly one single-byte token; each merge
// joins two usable tokens (not EOT, not empty) into exactly one token, and no pair repeats.
int make_tokenizer(const hsm::Model& M, hs_tokenizer* t) {
    const size_t V = M.vocab_ends.size();
    t->vocab = (uint32_t)V;
    t->eot = M.eot;
    t->n_ctx = (uint32_t)M.n_ctx;
    t->bytes = M.vocab_bytes;
    t->ends = M.vocab_ends;
    auto token = [&](size_t i) {
        const size_t a = i ? M.vocab_ends[i - 1] : 0;
        return std::string((const char*)M.vocab_bytes.data() + a, M.vocab_ends[i] - a);
    };
    std::unordered_map<std::string, int64_t> owner;  // bytes -> token, or -1 for two or more
    for (size_t i = 0; i < V; i++) {
        if (i == M.eot) continue;
        std::string b = token(i);
        if (b.empty()) continue;
        auto it = owner.find(b);
        if (it == owner.end()) owner.emplace(std::move(b), (int64_t)i);
        else it->second = -1;
    }
    for (int b = 0; b < 256; b++) {
        auto it = owner.find(std::string(1, (char)b));
        if (it == owner.end() || it->second < 0)
            return hs::host_fail(HS_MODEL, "no single token for byte " + std::to_string(b));
        t->byte_tokens[b] = (uint32_t)it->second;
    }
    t->merges.reserve(M.merges.size());
    for (size_t r = 0; r < M.merges.size(); r++) {
        const uint32_t l = M.merges[r].first, rt = M.merges[r].second;
        const std::string at = "merge rank " + std::to_string(r) + ": ";
        if (l >= V || rt >= V) return hs::host_fail(HS_MODEL, at + "a part is not in the vocabulary");
        if (l == M.eot || rt == M.eot || token(l).empty() || token(rt).empty())
            return hs::host_fail(HS_MODEL, at + "a part is <|endoftext|> or has no bytes");
        auto it = owner.find(token(l) + token(rt));
        if (it == owner.end()) return hs::host_fail(HS_MODEL, at + "no token has the joined bytes");
        if (it->second < 0) return hs::host_fail(HS_MODEL, at + "two or more tokens have the joined bytes");
        if (!t->merges.emplace(pair_key(l, rt), Merge{(uint32_t)r, (uint32_t)it->second}).second)
            return hs::host_fail(HS_MODEL, at + "the pair occurs two times");
    }
    return HS_OK;
}

}  // namespace

namespace hs {

// The tokenizer of a model whose file the runtime already parsed (hs_model_load).
int tokenizer_from_model(const hsm::Model& M, hs_tokenizer** out) {
    hs_tokenizer* t = new hs_tokenizer();
    const int rc = make_tokenizer(M, t);
    if (rc) {
        delete t;
        return rc;
    }
    *out = t;
    return HS_OK;
}

void tokenize(const hs_tokenizer* t, const uint8_t* data, size_t len, std::vector<uint32_t>& out) {
    t->encode(data, len, out);
}

bool model_file_info(const uint8_t* file, size_t len, uint32_t* vocab, uint32_t* eot, uint32_t* n_ctx,
                     std::string& err) {
    hsm::Model M;
    if (!file || !hsm::load_model(file, len, M, err)) return false;
    *vocab = (uint32_t)M.vocab;
    *eot = M.eot;
    *n_ctx = (uint32_t)M.n_ctx;
    return true;
}

void tokenizer_info(const hs_tokenizer* t, uint32_t* vocab, uint32_t* eot, uint32_t* n_ctx) {
    *vocab = t->vocab;
    *eot = t->eot;
    *n_ctx = t->n_ctx;
}

const uint8_t* token_bytes(const hs_tokenizer* t, uint32_t id, size_t* n) {
    if (id >= t->vocab) {
        *n = 0;
        return nullptr;
    }
    const size_t a = id ? t->ends[id - 1] : 0;
    *n = t->ends[id] - a;
    return t->bytes.data() + a;
}

bool tokens_restore(const hs_tokenizer* t, const uint32_t* tokens, size_t n, const uint8_t* data, size_t len) {
    size_t at = 0;
    for (size_t i = 0; i < n; i++) {
        const uint32_t id = tokens[i];
        if (id >= t->vocab || id == t->eot) return false;
        const size_t a = id ? t->ends[id - 1] : 0, e = t->ends[id];
        if (e == a || e - a > len - at || memcmp(t->bytes.data() + a, data + at, e - a) != 0) return false;
        at += e - a;
    }
    return at == len;
}

}  // namespace hs

extern "C" {

int hs_tokenizer_new(const uint8_t* file, size_t len, hs_tokenizer** out) {
    if (!file || !out) return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    hsm::Model M;
    std::string err;
    if (!hsm::load_model(file, len, M, err)) return hs::host_fail(HS_MODEL, "the model file is not valid: " + err);
    return hs::tokenizer_from_model(M, out);
}

void hs_tokenizer_free(hs_tokenizer* t) { delete t; }

int hs_tokenize(const hs_tokenizer* t, const uint8_t* data, size_t len, uint32_t* out, size_t cap, size_t* n) {
    if (!t || !n || (len && !data)) return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    std::vector<uint32_t> toks;
    toks.reserve(len);
    t->encode(data, len, toks);
    *n = toks.size();
    if (toks.size() > cap || (!out && !toks.empty()))
        return hs::host_fail(HS_BAD_ARGUMENT, "the output holds " + std::to_string(cap) + " tokens, " +
                                                  std::to_string(toks.size()) + " needed");
    if (!toks.empty()) memcpy(out, toks.data(), toks.size() * sizeof(uint32_t));
    return HS_OK;
}

int hs_tokenizer_pieces(const hs_tokenizer* t, const uint8_t* data, size_t len, uint64_t* ends, size_t cap,
                        size_t* n) {
    if (!t || !n || (len && !data)) return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    std::vector<uint64_t> e;
    std::vector<Char> ch;
    t->pieces(data, len, [&](size_t, size_t b, bool) { e.push_back(b); }, ch);
    *n = e.size();
    if (e.size() > cap || (!ends && !e.empty()))
        return hs::host_fail(HS_BAD_ARGUMENT, "the output holds " + std::to_string(cap) + " pieces");
    if (!e.empty()) memcpy(ends, e.data(), e.size() * sizeof(uint64_t));
    return HS_OK;
}

}  // extern "C"
