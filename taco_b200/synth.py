"""Seeded synthetic workloads of the benchmark (no network, no published weights here).

- `gpt2_hsm(seed)`: a GPT-2 124M-shaped model file (12 layers, d_model 768, 12 heads, FFN 3072,
  vocab 50257, ctx 1024) with float weights from seeded N(0, 0.02), biases 0, LayerNorm gamma 1
  and beta 0, converted to the HardShell .hsm integer format (version 1) with the rules of the
  reference converter (tools/convert/build.py of the reference): per-row symmetric int8 weights,
  activation scales from a float calibration pass, multipliers in [2^30, 2^31), the constants
  K = 48, J = 8, P = 30, exponent tables of 8192 entries with a unit of 2^-8, and 16-bit-input
  GELU tables. The reference converter needs the published GPT-2 files and exact rationals; this
  stand-in uses float64 numpy for the same rules, so its bytes are its own (the HardShell engine
  only needs a valid file).
- `zipf_text(...)`: seeded Zipf(s=1.1) text over a 5,000-word random lowercase vocabulary, space
  and newline separated (one line in about 12 words); `mixed_stream(...)` the large input of
  configs[4] (Zipf text, JSON-shaped key/number records and uniform random bytes in 64 KiB
  pieces).
- The synthetic vocabulary of GPT-2's size is byte-level BPE with merges, as the reference
  converter writes GPT-2's (crates/hardshell/src/hsm/merges.rs:1-20, the optional merges
  section): the 256 single bytes, every prefix of " w" and of "w" for the text words w, and the
  " w" prefixes of other words up to 50,256 tokens, then <|endoftext|>. Each multi-byte token t
  has the merge (t[:-1], t[-1]); the merges of the " w" tokens rank before those of the bare
  ones, so the tokenizer turns every " w" piece of the text into its one word token, and a bare
  word after a newline into one or a few tokens. `tokenize_text(...)` restates that BPE in Python
  for text of this alphabet only (a check of the product tokenizer, and the windows of the
  reference arm of the benchmark, which must not run this repository's engine).
- `text_windows(...)`: the token windows of the benchmark: consecutive n-token runs of the
  tokens of seeded Zipf text, so the bytes a window codes are bytes the fold would tokenize.
"""

from __future__ import annotations

import hashlib
import json
import os
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

N_LAYER, N_HEAD, D_MODEL, D_FF, VOCAB, N_CTX = 12, 12, 768, 3072, 50257, 1024


@dataclass(frozen=True)
class Shape:
    n_layer: int
    n_head: int
    d_model: int
    d_ff: int
    vocab: int
    n_ctx: int


GPT2 = Shape(N_LAYER, N_HEAD, D_MODEL, D_FF, VOCAB, N_CTX)
# A small model with GPT-2's head width (64) for the tests of the tensor-core attention.
MINI = Shape(2, 2, 128, 512, 1000, 512)
LN_K, LN_J, SOFTMAX_P = 48, 8, 30
TABLE_LEN, ATTN_EXP_E, LOGITS_EXP_E, DELTA = 8192, 30, 40, 2.0 ** -8
I32_MAX = 2**31 - 1
N_WORDS = 5000
CACHE = Path(__file__).resolve().parent / "_cache"


# ---- the synthetic vocabulary, its merges and the text ----

EOT_BYTES = b"<|endoftext|>"


def _words(seed: int, n: int) -> list[bytes]:
    """n distinct random lowercase words of 2 to 5 letters (the first N_WORDS are the text's)."""
    rng = np.random.default_rng(seed)
    letters = np.frombuffer(b"abcdefghijklmnopqrstuvwxyz", dtype=np.uint8)
    words: list[bytes] = []
    seen = set()
    while len(words) < n:
        w = letters[rng.integers(0, 26, int(rng.integers(2, 6)))].tobytes()
        if w not in seen:
            seen.add(w)
            words.append(w)
    return words


def vocabulary(seed: int = 0x7AC0, vocab: int = VOCAB) -> list[bytes]:
    """The token bytes, by id. For GPT-2's 50,257: 256 single bytes; the prefixes of " w" (length
    >= 2) and of "w" (length >= 2) of the N_WORDS text words; the " w" prefixes of further words
    until 50,256 tokens; <|endoftext|> last. Every token's bytes minus its last byte are a token,
    so each has a merge. For a smaller vocabulary: single bytes, " w" word tokens (no merges)."""
    if vocab != VOCAB:
        words = _words(seed, vocab - 257)
        return [bytes([b]) for b in range(256)] + [b" " + w for w in words] + [EOT_BYTES]
    words = _words(seed, 40_000)
    toks = [bytes([b]) for b in range(256)]
    seen = set(toks)

    def add(t: bytes):
        if t not in seen and len(toks) < VOCAB - 1:
            seen.add(t)
            toks.append(t)

    for w in words[:N_WORDS]:
        for i in range(1, len(w) + 1):
            add(b" " + w[:i])
    for w in words[:N_WORDS]:
        for i in range(2, len(w) + 1):
            add(w[:i])
    for w in words[N_WORDS:]:
        for i in range(1, len(w) + 1):
            add(b" " + w[:i])
    assert len(toks) == VOCAB - 1
    toks.append(EOT_BYTES)
    return toks


def merges(vocab: list[bytes]) -> list[tuple[int, int]]:
    """The BPE merges in rank order: (id of t[:-1], id of t[-1:]) for each multi-byte token t but
    <|endoftext|>; the tokens that start with a space first, then the others, each group in id
    order (a prefix before its extensions). Empty for a vocabulary whose tokens are not closed
    under dropping the last byte (the small test vocabularies)."""
    ids = {t: i for i, t in enumerate(vocab)}
    out_sp, out_bare = [], []
    for i, t in enumerate(vocab):
        if len(t) < 2 or t == EOT_BYTES:
            continue
        left = ids.get(t[:-1])
        if left is None:
            return []
        (out_sp if t[:1] == b" " else out_bare).append((left, ids[t[-1:]]))
    return out_sp + out_bare


def text_word_ids(vocab: list[bytes]) -> np.ndarray:
    """The ids of the " w" tokens of the N_WORDS text words, in Zipf rank order."""
    ids = {t: i for i, t in enumerate(vocab)}
    return np.array([ids[b" " + w] for w in _words(0x7AC0, N_WORDS)], dtype=np.uint32)


def _zipf_draw(rng, n: int) -> np.ndarray:
    """n word indices of the Zipf(1.1) law over N_WORDS (inverse CDF of one uniform draw each)."""
    p = np.arange(1, N_WORDS + 1, dtype=np.float64) ** -1.1
    cdf = np.cumsum(p / p.sum())
    return np.minimum(np.searchsorted(cdf, rng.random(n), side="right"), N_WORDS - 1)


def zipf_text(n_bytes: int, seed: int) -> bytes:
    """About n_bytes (at least) of seeded Zipf(1.1) text over the N_WORDS text words, each word
    after a space, or after a newline with probability 1/12; the text starts with a word."""
    rng = np.random.default_rng(seed)
    words = _words(0x7AC0, N_WORDS)
    lens = np.array([len(w) for w in words], dtype=np.int64)
    letters = np.zeros((N_WORDS, 5), dtype=np.uint8)
    for i, w in enumerate(words):
        letters[i, :len(w)] = np.frombuffer(w, dtype=np.uint8)
    out, total = [], 0
    while total < n_bytes:
        n = min(1 << 20, max(1024, (n_bytes - total) // 4 + 16))
        idx = _zipf_draw(rng, n)
        nl = rng.random(n) < 1.0 / 12
        wl = lens[idx] + 1  # the separator, then the word
        starts = np.concatenate([[0], np.cumsum(wl)[:-1]])
        chunk = np.empty(int(wl.sum()), dtype=np.uint8)
        chunk[starts] = np.where(nl, ord("\n"), ord(" "))
        for k in range(5):
            m = lens[idx] > k
            chunk[starts[m] + 1 + k] = letters[idx[m], k]
        out.append(chunk.tobytes())
        total += chunk.size
    return b"".join(out)[1:]


def json_records(n_bytes: int, seed: int) -> bytes:
    """About n_bytes (at least) of JSON-shaped records, one per line: 1 to 6 "key": number pairs,
    keys from the text words (Zipf), numbers uniform integers in [-10^6, 10^6]; e.g.
    {"abc": -12, "qz": 40571}."""
    rng = np.random.default_rng(seed)
    words = _words(0x7AC0, N_WORDS)
    # Each key as the bytes '"word": ' (at most 9 bytes).
    keys = [b'"' + w + b'": ' for w in words]
    klen = np.array([len(k) for k in keys], dtype=np.int64)
    kbytes = np.zeros((N_WORDS, 9), dtype=np.uint8)
    for i, k in enumerate(keys):
        kbytes[i, :len(k)] = np.frombuffer(k, dtype=np.uint8)
    out, total = [], 0
    while total < n_bytes:
        n = max(256, (n_bytes - total) // 40 + 16)  # records
        c = rng.integers(1, 7, n)
        P = int(c.sum())
        kid = _zipf_draw(rng, P)
        num = rng.integers(-10**6, 10**6 + 1, P)
        mag = np.abs(num)
        ndig = np.ones(P, dtype=np.int64)
        for t in range(1, 7):
            ndig += mag >= 10 ** t
        neg = (num < 0).astype(np.int64)
        first = np.zeros(P, dtype=bool)
        first[np.concatenate([[0], np.cumsum(c)[:-1]])] = True
        last = np.zeros(P, dtype=bool)
        last[np.cumsum(c) - 1] = True
        # A pair: "{" if first, else ", "; the key; "-" if negative; the digits; "}\n" if last.
        pre = np.where(first, 1, 2)
        plen = pre + klen[kid] + neg + ndig + np.where(last, 2, 0)
        start = np.concatenate([[0], np.cumsum(plen)[:-1]])
        buf = np.empty(int(plen.sum()), dtype=np.uint8)
        buf[start[first]] = ord("{")
        nf = ~first
        buf[start[nf]] = ord(",")
        buf[start[nf] + 1] = ord(" ")
        at = start + pre
        for k in range(9):
            m = klen[kid] > k
            buf[at[m] + k] = kbytes[kid[m], k]
        at = at + klen[kid]
        buf[at[neg == 1]] = ord("-")
        at = at + neg
        for k in range(7):  # digit k from the left
            m = ndig > k
            e = ndig[m] - 1 - k
            buf[at[m] + k] = ord("0") + (mag[m] // (10 ** e)) % 10
        at = at + ndig
        buf[at[last]] = ord("}")
        buf[at[last] + 1] = ord("\n")
        out.append(buf.tobytes())
        total += buf.size
    return b"".join(out)


def mixed_kinds(n: int, seed: int = 4) -> np.ndarray:
    """The kinds of the n pieces of mixed_stream: 0 Zipf text (70 %), 1 JSON records (20 %),
    2 uniform random bytes (the rest), in a seeded order."""
    rng = np.random.default_rng(seed)
    kinds = np.array([0] * (n * 7 // 10) + [1] * (n * 2 // 10), dtype=np.int8)
    kinds = np.concatenate([kinds, np.full(n - kinds.size, 2, np.int8)])
    rng.shuffle(kinds)
    return kinds


def mixed_stream(n_bytes: int = 256 << 20, seed: int = 4, piece: int = 64 << 10) -> bytes:
    """n_bytes of seeded input in pieces of `piece` bytes, 70 % Zipf text, 20 %
    JSON-shaped key/number records and 10 % uniform random bytes (exact counts of pieces, in a
    seeded order: mixed_kinds)."""
    n = n_bytes // piece
    kinds = mixed_kinds(n, seed)
    rng = np.random.default_rng(seed + 3)
    counts = np.bincount(kinds, minlength=3)
    text = zipf_text(int(counts[0]) * piece, seed + 1)
    js = json_records(int(counts[1]) * piece, seed + 2)
    rnd = rng.integers(0, 256, int(counts[2]) * piece, dtype=np.uint8).tobytes()
    src = [text, js, rnd]
    at = [0, 0, 0]
    out = bytearray()
    for k in kinds.tolist():
        out += src[k][at[k]:at[k] + piece]
        at[k] += piece
    return bytes(out)


def tokenize_text(text: bytes, vocab: list[bytes], merge_list: list[tuple[int, int]]) -> np.ndarray:
    """Byte-level BPE of text made of lowercase words, spaces and newlines only (zipf_text): the
    GPT-2 pattern cuts it into " w", "w" and newline pieces (crates/taco/src/tokenizer/
    pretokenize.rs), and each piece merges the adjacent pair of lowest rank first, every place of
    that pair from the left, until no pair has a rank (bpe.rs). Each distinct piece is merged
    once."""
    import re

    ids = {t: i for i, t in enumerate(vocab)}
    rank = {pair: r for r, pair in enumerate(merge_list)}
    joined = {(a, b): ids[vocab[a] + vocab[b]] for a, b in merge_list}
    memo: dict[bytes, list[int]] = {}

    def bpe(piece: bytes) -> list[int]:
        t = [ids[piece[i:i + 1]] for i in range(len(piece))]
        while len(t) > 1:
            best = min(((rank.get((t[i], t[i + 1]), 1 << 62), i) for i in range(len(t) - 1)))[0]
            if best == 1 << 62:
                break
            pair = merge_list[best]
            out, i = [], 0
            while i < len(t):
                if i + 1 < len(t) and (t[i], t[i + 1]) == pair:
                    out.append(joined[pair])
                    i += 2
                else:
                    out.append(t[i])
                    i += 1
            t = out
        return t

    pieces = re.findall(rb"\n+| ?[a-z]+| +", text)
    assert sum(len(x) for x in pieces) == len(text), "text outside the alphabet of zipf_text"
    out: list[int] = []
    for pc in pieces:
        got = memo.get(pc)
        if got is None:
            got = memo[pc] = bpe(pc)
        out.extend(got)
    return np.array(out, dtype=np.uint32)


def text_windows(n_windows: int, window: int, seed: int) -> np.ndarray:
    """[n_windows, window] token ids: consecutive runs of the tokens of seeded Zipf text
    (zipf_text, tokenize_text with the GPT-2-sized synthetic vocabulary and its merges)."""
    vocab = vocabulary()
    need = n_windows * window
    text = zipf_text(int(need * 4.7) + 4096, seed)
    toks = tokenize_text(text, vocab, merges(vocab))
    while toks.size < need:
        text += b" " + zipf_text(int((need - toks.size) * 5) + 4096, seed + toks.size)
        toks = tokenize_text(text, vocab, merges(vocab))
    return toks[:need].reshape(n_windows, window)


def token_lengths(vocab: list[bytes]) -> np.ndarray:
    return np.array([len(t) for t in vocab], dtype=np.int64)


# ---- the float model and its calibration ----

def _gelu(x):
    return 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))


def _ln(x, g, b):
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + 1e-5) * g + b


def float_model(seed: int, sh: Shape = GPT2) -> dict:
    rng = np.random.default_rng(seed)
    n = lambda *s: rng.normal(0.0, 0.02, s).astype(np.float32)  # noqa: E731
    d, f = sh.d_model, sh.d_ff
    m = {"wte": n(sh.vocab, d), "wpe": n(sh.n_ctx, d), "blocks": [], "shape": sh}
    for _ in range(sh.n_layer):
        m["blocks"].append({"attn_w": n(3 * d, d), "proj_w": n(d, d), "fc_w": n(f, d), "mlp_w": n(d, f)})
    return m


def calibrate(fm: dict, seed: int, seqs: int = 2, length: int = 256) -> dict:
    """The largest |x| of each activation site, and the residual max and smallest row std."""
    sh: Shape = fm["shape"]
    rng = np.random.default_rng(seed ^ 0xCA1)
    ranges: dict[str, float] = {}
    res_max, row_std = 0.0, np.inf
    hd = sh.d_model // sh.n_head
    length = min(length, sh.n_ctx)
    one = np.ones(sh.d_model, np.float32)
    zero = np.zeros(sh.d_model, np.float32)

    def see(k, v):
        ranges[k] = max(ranges.get(k, 0.0), float(np.abs(v).max()))

    for _ in range(seqs):
        toks = rng.integers(0, sh.vocab - 1, length)
        x = fm["wte"][toks] + fm["wpe"][:length]
        for l, b in enumerate(fm["blocks"]):
            res_max = max(res_max, float(np.abs(x).max()))
            row_std = min(row_std, float(x.std(-1).min()))
            a = _ln(x, one, zero)
            see(f"h.{l}.ln_1", a)
            qkv = a @ b["attn_w"].T
            q, k, v = np.split(qkv, 3, axis=-1)
            see(f"h.{l}.q", q)
            see(f"h.{l}.k", k)
            see(f"h.{l}.v", v)
            att = np.zeros_like(q)
            mask = np.triu(np.full((length, length), -np.inf, np.float32), 1)
            for h in range(sh.n_head):
                sl = slice(h * hd, (h + 1) * hd)
                s = q[:, sl] @ k[:, sl].T / np.sqrt(hd) + mask
                s = np.exp(s - s.max(-1, keepdims=True))
                s /= s.sum(-1, keepdims=True)
                att[:, sl] = s @ v[:, sl]
            see(f"h.{l}.att", att)
            x = x + att @ b["proj_w"].T
            a = _ln(x, one, zero)
            see(f"h.{l}.ln_2", a)
            f = a @ b["fc_w"].T
            see(f"h.{l}.fc", f)
            g = _gelu(f)
            see(f"h.{l}.gelu", g)
            x = x + g @ b["mlp_w"].T
        res_max = max(res_max, float(np.abs(x).max()))
        row_std = min(row_std, float(x.std(-1).min()))
        see("ln_f", _ln(x, one, zero))
    ranges["res_max"] = res_max
    ranges["row_std_min"] = row_std
    return ranges


# ---- the conversion rules (tools/convert/build.py and exact.py of the reference) ----

def quantise_rows(w: np.ndarray, qmax: int = 127) -> tuple[np.ndarray, np.ndarray]:
    w = np.asarray(w, np.float64)
    mx = np.abs(w).max(axis=1)
    scale = np.where(mx > 0, mx / qmax, 1.0)
    q = np.clip(np.rint(w / scale[:, None]), -qmax, qmax).astype(np.int64)
    return q, scale


def quant_mult_rows(ratios) -> tuple[np.ndarray, int]:
    r = np.asarray(ratios, np.float64)
    mx = float(r.max())
    assert 0 < mx < I32_MAX and r.min() >= 0
    s = 0
    while s < 126 and mx * 2.0 ** (s + 1) < I32_MAX:
        s += 1
    m = np.rint(r * 2.0 ** s)
    assert m.max() <= I32_MAX
    return m.astype(np.int32), s


def quant_mult(ratio: float) -> tuple[int, int]:
    m, s = quant_mult_rows([ratio])
    return int(m[0]), s


def exp_table(e: int) -> np.ndarray:
    i = np.arange(TABLE_LEN, dtype=np.float64)
    t = np.rint(2.0 ** e * np.exp(-i * DELTA))
    t[0] = 2.0 ** e
    return t


def gelu_table(s_in: float, s_out: float) -> np.ndarray:
    x = np.arange(-32768, 32768, dtype=np.float64) * s_in
    return np.clip(np.rint(_gelu(x) / s_out), -127, 127).astype(np.int8)


def gelu_table16(s_in: float, s_out: float) -> np.ndarray:
    """The i16-output GELU table of a version 2 model (crates/hardshell/src/gelu.rs)."""
    x = np.arange(-32768, 32768, dtype=np.float64) * s_in
    return np.clip(np.rint(_gelu(x) / s_out), -32767, 32767).astype(np.int16)


# A version 2 ("wide") synthetic model: a 16-bit final LayerNorm (ln_f_bits = 16), LayerNorm
# betas with BETA_FRAC fractional bits, and 16-bit GELU outputs in the even layers.
BETA_FRAC = 4


def build_tensors(fm: dict, rg: dict, wide: bool = False) -> list[tuple[str, str, np.ndarray, int | None]]:
    """(name, dtype, values, shift) in the order of crates/hardshell/src/gpt2/mod.rs. `wide`: the
    version 2 rules (16-bit ln_f, 16-bit GELU in the even layers, betas with BETA_FRAC
    fractional bits)."""
    out: list[tuple[str, str, np.ndarray, int | None]] = []
    brng = np.random.default_rng(fm.get("seed", 0) + 99)
    sh: Shape = fm["shape"]
    D_MODEL, D_FF, N_HEAD = sh.d_model, sh.d_ff, sh.n_head  # noqa: N806
    res = min(rg["res_max"] / 2 ** 24, rg["row_std_min"] / 2 ** 12.5)
    site = lambda k, qmax=127: rg[k] / qmax  # noqa: E731
    s_lnf = site("ln_f") / (256 if wide else 1)
    wq, ws = quantise_rows(fm["wte"])
    out.append(("wte", "i8", wq.astype(np.int8), None))
    m, s = quant_mult_rows(ws / res)
    out.append(("wte.rescale_embed", "i32", m, s))
    m, s = quant_mult_rows(ws * s_lnf / DELTA)
    out.append(("wte.rescale_logits", "i32", m, s))
    pq, ps = quantise_rows(fm["wpe"])
    out.append(("wpe", "i8", pq.astype(np.int8), None))
    m, s = quant_mult_rows(ps / res)
    out.append(("wpe.rescale", "i32", m, s))

    def layernorm(prefix, s_out):
        gq, gs = quantise_rows(np.ones((1, D_MODEL)), 32767)
        out.append((f"{prefix}.g", "i16", gq.reshape(-1).astype(np.int16), None))
        if wide:
            # Betas of about 0.05 of the output scale, in units of 2^-BETA_FRAC of an output step.
            beta = np.rint(brng.normal(0.0, 0.05 / s_out, D_MODEL) * 2 ** BETA_FRAC)
            out.append((f"{prefix}.b", "i32", beta.astype(np.int32), None))
        else:
            out.append((f"{prefix}.b", "i32", np.zeros(D_MODEL, np.int32), None))
        mm, ss = quant_mult(gs[0] / (2.0 ** (LN_K - LN_J) * s_out))
        out.append((f"{prefix}.rescale", "i32", np.array([mm], np.int32), ss))

    def linear(prefix, w, s_in, s_out):
        q, ws_ = quantise_rows(w)
        out.append((f"{prefix}.w", "i8", q.astype(np.int8), None))
        out.append((f"{prefix}.b", "i32", np.zeros(w.shape[0], np.int32), None))
        mm, ss = quant_mult_rows(s_in * ws_ / np.asarray(s_out))
        out.append((f"{prefix}.rescale", "i32", mm, ss))

    hd = D_MODEL // N_HEAD
    for l, b in enumerate(fm["blocks"]):
        p = f"h.{l}"
        layernorm(f"{p}.ln_1", site(f"{p}.ln_1"))
        sq, sk, sv = site(f"{p}.q"), site(f"{p}.k"), site(f"{p}.v")
        qkv_out = np.concatenate([np.full(D_MODEL, sq), np.full(D_MODEL, sk), np.full(D_MODEL, sv)])
        linear(f"{p}.attn.c_attn", b["attn_w"], site(f"{p}.ln_1"), qkv_out)
        mm, ss = quant_mult(sq * sk / DELTA / np.sqrt(hd))
        out.append((f"{p}.attn.score.rescale", "i32", np.array([mm], np.int32), ss))
        mm, ss = quant_mult(sv / (2.0 ** SOFTMAX_P * site(f"{p}.att")))
        out.append((f"{p}.attn.out.rescale", "i32", np.array([mm], np.int32), ss))
        linear(f"{p}.attn.c_proj", b["proj_w"], site(f"{p}.att"), np.full(D_MODEL, res))
        layernorm(f"{p}.ln_2", site(f"{p}.ln_2"))
        s_fc = site(f"{p}.fc", 32767)
        linear(f"{p}.mlp.c_fc", b["fc_w"], site(f"{p}.ln_2"), np.full(D_FF, s_fc))
        if wide and l % 2 == 0:
            s_g = site(f"{p}.gelu") / 256
            out.append((f"{p}.mlp.gelu", "i16", gelu_table16(s_fc, s_g), None))
        else:
            s_g = site(f"{p}.gelu")
            out.append((f"{p}.mlp.gelu", "i8", gelu_table(s_fc, s_g), None))
        linear(f"{p}.mlp.c_proj", b["mlp_w"], s_g, np.full(D_MODEL, res))
    layernorm("ln_f", s_lnf)
    out.append(("attn_exp", "i32", exp_table(ATTN_EXP_E).astype(np.int32), None))
    out.append(("logits_exp", "u64", exp_table(LOGITS_EXP_E).astype(np.uint64), None))
    return out, res


def write_hsm(tensors, vocab: list[bytes], eps: int, sh: Shape = GPT2, wide: bool = False) -> bytes:
    """The .hsm layout (crates/hardshell/src/hsm/mod.rs:1-120): preamble, compact JSON header,
    vocabulary, the merges section when the vocabulary has merges (two u32 ids per merge in rank
    order, at the 64-byte boundary after the vocabulary: hsm/merges.rs:1-20), and tensors at
    64-byte boundaries with zero padding."""
    vocab_sec = b"".join(struct.pack("<H", len(t)) + t for t in vocab)
    merge_sec = b"".join(struct.pack("<II", a, b) for a, b in merges(vocab))
    dt = {"i8": np.int8, "i16": np.int16, "i32": np.int32, "u64": np.uint64}
    blobs = [(n, d, np.ascontiguousarray(v, dtype=dt[d]).astype(np.dtype(dt[d]).newbyteorder("<")), s)
             for n, d, v, s in tensors]
    align = lambda x: (x + 63) & ~63  # noqa: E731
    hlen = 4096
    while True:
        cursor = align(16 + hlen)
        voff = cursor
        cursor = voff + len(vocab_sec)
        moff = align(cursor)
        if merge_sec:
            cursor = moff + len(merge_sec)
        entries = []
        for n, d, v, s in blobs:
            off = align(cursor)
            e = {"name": n, "dtype": d, "shape": list(v.shape), "offset": off, "length": v.nbytes}
            if s is not None:
                e["shift"] = int(s)
            entries.append(e)
            cursor = off + v.nbytes
        header = {
            "model": {"architecture": "gpt2", "n_layer": sh.n_layer, "n_head": sh.n_head, "d_model": sh.d_model,
                      "d_ff": sh.d_ff, "vocab_size": sh.vocab, "n_ctx": sh.n_ctx, "eot_token": sh.vocab - 1,
                      "constants": dict({"ln_k": LN_K, "ln_j": LN_J, "ln_eps": eps, "softmax_p": SOFTMAX_P},
                                        **({"ln_f_bits": 16, "ln_beta_frac": BETA_FRAC} if wide else {}))},
            "vocabulary": {"offset": voff, "length": len(vocab_sec)},
            **({"merges": {"offset": moff, "length": len(merge_sec)}} if merge_sec else {}),
            "tensors": entries,
        }
        text = json.dumps(header, separators=(",", ":")).encode()
        if len(text) <= hlen:
            text += b" " * (hlen - len(text))
            break
        hlen = len(text)
    out = bytearray(b"HSHLMDL\0" + struct.pack("<II", 2 if wide else 1, hlen) + text)
    out += bytes(align(len(out)) - len(out))
    out += vocab_sec
    if merge_sec:
        out += bytes(moff - len(out))
        out += merge_sec
    for (n, d, v, s), e in zip(blobs, entries):
        out += bytes(e["offset"] - len(out))
        out += v.tobytes()
    return bytes(out)


def gpt2_hsm(seed: int = 124, cache: bool = True, shape: Shape = GPT2, wide: bool = False) -> bytes:
    """The synthetic GPT-2 model file for `seed` and `shape` (GPT-2 124M by default; cached under
    taco_b200/_cache). `wide`: a version 2 file (16-bit ln_f and GELU, fractional betas)."""
    tag = "gpt2_124m_bpe" if shape == GPT2 else "gpt2_{}l{}h{}d{}f{}v{}c".format(*vars(shape).values())
    tag += "_v2" if wide else ""
    path = CACHE / f"{tag}_seed{seed}.hsm"
    if cache and path.exists():
        return path.read_bytes()
    fm = float_model(seed, shape)
    rg = calibrate(fm, seed)
    tensors, res = build_tensors(fm, rg, wide)
    eps = max(1, int(round(1e-5 / (res * res) * 2 ** (2 * LN_J))))
    data = write_hsm(tensors, vocabulary(vocab=shape.vocab), eps, shape, wide)
    if cache:
        CACHE.mkdir(exist_ok=True)
        tmp = path.with_suffix(f".{os.getpid()}.tmp")  # one per process: ranks may build it at once
        tmp.write_bytes(data)
        tmp.replace(path)
    return data


def describe(data: bytes) -> str:
    return f"{len(data)} bytes, sha256 {hashlib.sha256(data).hexdigest()[:16]}"
