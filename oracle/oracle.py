"""TEST INFRASTRUCTURE ONLY: ctypes binding of the CPU oracle (oracle/_build/libhsoracle.so).

The oracle is a C++ restatement of the reference CPU engine (crates/hardshell) and coder
(crates/taco-coder). Only tests/, `__graft_entry__.smoke()` and the CPU-baseline leg of
bench.py use it, and only as the checker or the timed CPU baseline. The GPU product
(taco_b200) never imports it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libhsoracle.so"

_lib = None


def build() -> Path:
    """Compiles the oracle with its Makefile (g++ only)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build()
    L = ctypes.CDLL(str(LIB_PATH))
    vp, sz, u8p = ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint8)
    L.hso_model_load.restype = vp
    L.hso_model_load.argtypes = [ctypes.c_char_p, sz, ctypes.c_char_p, sz]
    L.hso_model_free.argtypes = [vp]
    L.hso_model_dims.argtypes = [vp, ctypes.c_void_p]
    L.hso_vocab_token.argtypes = [vp, ctypes.c_uint32, ctypes.POINTER(u8p), ctypes.POINTER(sz)]
    L.hso_merges.argtypes = [vp, ctypes.c_void_p, sz]
    L.hso_session_new.restype = vp
    L.hso_session_new.argtypes = [vp, ctypes.c_uint16]
    L.hso_session_free.argtypes = [vp]
    L.hso_session_reset.argtypes = [vp]
    L.hso_session_position.argtypes = [vp]
    L.hso_session_step.argtypes = [vp, ctypes.c_uint32, ctypes.c_void_p]
    L.hso_session_coded.argtypes = [vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32,
                                    ctypes.c_void_p]
    L.hso_from_weights.argtypes = [ctypes.c_void_p, sz, ctypes.c_uint32, ctypes.c_void_p]
    L.hso_answer.argtypes = [ctypes.c_void_p, sz, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64,
                             ctypes.c_void_p]
    L.hso_mix_stats.argtypes = [ctypes.c_void_p, sz, ctypes.c_uint32, ctypes.c_void_p]
    L.hso_mix_weights.argtypes = [ctypes.c_void_p, sz, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p]
    L.hso_encode_block.argtypes = [vp, ctypes.c_uint16, ctypes.c_void_p, sz, ctypes.c_void_p, sz,
                                   ctypes.POINTER(sz)]
    L.hso_decode_block.argtypes = [vp, ctypes.c_uint16, ctypes.c_char_p, sz, ctypes.c_uint32, ctypes.c_void_p,
                                   sz, ctypes.c_void_p, sz, ctypes.POINTER(sz)]
    L.hso_enc_new.restype = vp
    L.hso_enc_free.argtypes = [vp]
    L.hso_enc_interval.argtypes = [vp, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, ctypes.c_uint32]
    L.hso_enc_bit.argtypes = [vp, ctypes.c_uint32, ctypes.c_int]
    L.hso_enc_min_final_len.restype = sz
    L.hso_enc_min_final_len.argtypes = [vp]
    L.hso_enc_finish.restype = sz
    L.hso_enc_finish.argtypes = [vp, ctypes.c_void_p, sz]
    L.hso_dec_new.restype = vp
    L.hso_dec_new.argtypes = [ctypes.c_char_p, sz]
    L.hso_dec_free.argtypes = [vp]
    L.hso_dec_target.restype = ctypes.c_uint64
    L.hso_dec_target.argtypes = [vp, ctypes.c_uint32]
    L.hso_dec_interval.argtypes = [vp, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, ctypes.c_uint32]
    L.hso_dec_table.restype = ctypes.c_uint32
    L.hso_dec_table.argtypes = [vp, ctypes.c_void_p, sz, ctypes.c_uint32]
    L.hso_dec_bit.argtypes = [vp, ctypes.c_uint32]
    L.hso_layernorm_rows.argtypes = [vp, ctypes.c_int, ctypes.c_void_p, sz, ctypes.c_void_p, ctypes.c_void_p]
    L.hso_fast_new.restype = vp
    L.hso_fast_new.argtypes = [vp, ctypes.c_int, ctypes.c_uint16]
    L.hso_fast_free.argtypes = [vp]
    L.hso_fast_reset.argtypes = [vp, ctypes.c_int]
    L.hso_fast_position.argtypes = [vp, ctypes.c_int]
    L.hso_fast_run.argtypes = [vp, ctypes.c_void_p, ctypes.c_void_p, sz, ctypes.c_void_p, ctypes.c_void_p,
                               ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    L.hso_fast_run_lanes.argtypes = [vp, ctypes.c_void_p, ctypes.c_void_p, sz, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    _lib = L
    return L


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


DIM_NAMES = ["n_layer", "n_head", "d_model", "d_ff", "head_dim", "vocab", "n_ctx", "eot", "ln_f_bits",
             "ln_beta_frac", "is_wide", "version", "attn_exp_len", "logits_exp_len", "softmax_p", "n_merges"]


class OracleError(RuntimeError):
    pass


class Model:
    """crates/hardshell/src/gpt2/model.rs Model, loaded by the oracle."""

    def __init__(self, data: bytes):
        L = lib()
        err = ctypes.create_string_buffer(512)
        self._data = bytes(data)
        self.h = L.hso_model_load(self._data, len(self._data), err, 512)
        if not self.h:
            raise OracleError(err.value.decode())
        out = np.zeros(16, dtype=np.int64)
        L.hso_model_dims(self.h, _ptr(out))
        self.dims = dict(zip(DIM_NAMES, (int(v) for v in out)))
        self.vocab = self.dims["vocab"]
        self.n_ctx = self.dims["n_ctx"]
        self.eot = self.dims["eot"]

    def __del__(self):
        if getattr(self, "h", None):
            lib().hso_model_free(self.h)
            self.h = None

    def token_bytes(self, t: int) -> bytes:
        p = ctypes.POINTER(ctypes.c_uint8)()
        n = ctypes.c_size_t()
        if lib().hso_vocab_token(self.h, t, ctypes.byref(p), ctypes.byref(n)):
            raise OracleError("token out of range")
        return ctypes.string_at(p, n.value)

    def merges(self) -> list[tuple[int, int]]:
        n = self.dims["n_merges"]
        buf = np.zeros(2 * max(n, 1), dtype=np.uint32)
        lib().hso_merges(self.h, _ptr(buf), buf.size)
        return [(int(buf[2 * i]), int(buf[2 * i + 1])) for i in range(n)]

    def layernorm(self, which: int, x: np.ndarray, wide: bool = False) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.int32)
        rows = x.shape[0]
        if wide:
            out = np.zeros_like(x, dtype=np.int16)
            lib().hso_layernorm_rows(self.h, which, _ptr(x), rows, None, _ptr(out))
        else:
            out = np.zeros_like(x, dtype=np.int8)
            lib().hso_layernorm_rows(self.h, which, _ptr(x), rows, _ptr(out), None)
        return out


class Session:
    """crates/hardshell/src/gpt2/reference.rs ReferenceSession."""

    def __init__(self, model: Model, overlap: int = 0):
        self.model = model
        self.h = lib().hso_session_new(model.h, overlap)

    def __del__(self):
        if getattr(self, "h", None):
            lib().hso_session_free(self.h)
            self.h = None

    @property
    def position(self) -> int:
        return lib().hso_session_position(self.h)

    def reset(self):
        lib().hso_session_reset(self.h)

    def step(self, token: int) -> np.ndarray:
        w = np.zeros(self.model.vocab, dtype=np.uint64)
        rc = lib().hso_session_step(self.h, token, _ptr(w))
        if rc:
            raise OracleError(f"step failed: {rc}")
        return w

    def start_block(self) -> np.ndarray:
        self.reset()
        return self.step(self.model.eot)

    def coded(self, token: int, kind: int, value: int, bits: int = 32) -> tuple[int, int, int]:
        out = np.zeros(3, dtype=np.uint64)
        rc = lib().hso_session_coded(self.h, token, kind, value, bits, _ptr(out))
        if rc:
            raise OracleError(f"coded step failed: {rc}")
        return int(out[0]), int(out[1]), int(out[2])


def from_weights(w: np.ndarray, bits: int) -> np.ndarray:
    """freq.rs:103 FreqTable::from_weights: the cumulative starts (u32)."""
    w = np.ascontiguousarray(w, dtype=np.uint64)
    starts = np.zeros(w.size, dtype=np.uint32)
    rc = lib().hso_from_weights(_ptr(w), w.size, bits, _ptr(starts))
    if rc:
        raise OracleError(f"from_weights failed: {rc}")
    return starts


def answer(w: np.ndarray, bits: int, kind: int, value: int) -> tuple[int, int, int]:
    w = np.ascontiguousarray(w, dtype=np.uint64)
    out = np.zeros(3, dtype=np.uint64)
    rc = lib().hso_answer(_ptr(w), w.size, bits, kind, value, _ptr(out))
    if rc:
        raise OracleError(f"answer failed: {rc}")
    return int(out[0]), int(out[1]), int(out[2])


MIX_NONE = 0xFFFFFFFF  # crates/hardshell-cuda/src/mixed.rs:31: an input without a prediction
MIX_PLAIN = 0xFFFFFFFE  # mixed.rs:104: the table of GPT-2 alone


def mix_stats(w: np.ndarray, p: int) -> tuple[int, int, int]:
    """taco-match mixer.rs:276-287, pass 1 of Mixer::mix: (W, w[p], top)."""
    w = np.ascontiguousarray(w, dtype=np.uint64)
    out = np.zeros(3, dtype=np.uint64)
    rc = lib().hso_mix_stats(_ptr(w), w.size, p, _ptr(out))
    if rc:
        raise OracleError(f"mix_stats failed: {rc}")
    return int(out[0]), int(out[1]), int(out[2])


def mix_weights(w: np.ndarray, p: int, q: int = 0) -> np.ndarray:
    """The weights of Mixer::mix (mixer.rs:265-269 rule 1, :491-516 apply) for the table word p
    (a token, MIX_NONE or MIX_PLAIN) and the mixer probability q in 1..=65535."""
    w = np.ascontiguousarray(w, dtype=np.uint64)
    out = np.zeros(w.size, dtype=np.uint64)
    rc = lib().hso_mix_weights(_ptr(w), w.size, p, q, _ptr(out))
    if rc:
        raise OracleError(f"mix_weights failed: {rc}")
    return out


def encode_block(model: Model, tokens, overlap: int = 0) -> bytes:
    t = np.ascontiguousarray(tokens, dtype=np.uint32)
    cap = 64 + 8 * max(1, t.size)
    out = np.zeros(cap, dtype=np.uint8)
    n = ctypes.c_size_t()
    rc = lib().hso_encode_block(model.h, overlap, _ptr(t), t.size, _ptr(out), cap, ctypes.byref(n))
    if rc:
        raise OracleError(f"encode_block failed: {rc}")
    return out[: n.value].tobytes()


def decode_block(model: Model, payload: bytes, original_len: int, overlap: int = 0) -> tuple[bytes, list[int]]:
    out = np.zeros(max(1, original_len), dtype=np.uint8)
    toks = np.zeros(max(1, original_len), dtype=np.uint32)
    n = ctypes.c_size_t()
    rc = lib().hso_decode_block(model.h, overlap, payload, len(payload), original_len, _ptr(out), out.size,
                                _ptr(toks), toks.size, ctypes.byref(n))
    if rc:
        raise OracleError(f"decode_block failed: {rc}")
    return out[:original_len].tobytes(), [int(v) for v in toks[: n.value]]


class Encoder:
    def __init__(self):
        self.h = lib().hso_enc_new()

    def __del__(self):
        if getattr(self, "h", None):
            lib().hso_enc_free(self.h)

    def interval(self, start: int, freq: int, is_last: bool, bits: int):
        lib().hso_enc_interval(self.h, start, freq, int(is_last), bits)

    def bit(self, p1: int, bit: bool):
        lib().hso_enc_bit(self.h, p1, int(bit))

    def min_final_len(self) -> int:
        return lib().hso_enc_min_final_len(self.h)

    def finish(self) -> bytes:
        cap = 1 << 20
        buf = np.zeros(cap, dtype=np.uint8)
        n = lib().hso_enc_finish(self.h, _ptr(buf), cap)
        assert n <= cap
        return buf[:n].tobytes()


class Decoder:
    def __init__(self, data: bytes):
        self.h = lib().hso_dec_new(data, len(data))

    def __del__(self):
        if getattr(self, "h", None):
            lib().hso_dec_free(self.h)

    def target(self, bits: int) -> int:
        return lib().hso_dec_target(self.h, bits)

    def interval(self, start: int, freq: int, is_last: bool, bits: int) -> bool:
        return lib().hso_dec_interval(self.h, start, freq, int(is_last), bits) == 0

    def table(self, starts: np.ndarray, bits: int) -> int:
        starts = np.ascontiguousarray(starts, dtype=np.uint32)
        return lib().hso_dec_table(self.h, _ptr(starts), starts.size, bits)

    def bit(self, p1: int) -> bool:
        return lib().hso_dec_bit(self.h, p1) == 1


class FastBatch:
    """The fast CPU path: slots in chunks of 32 rows, SIMD dot products, all host threads."""

    def __init__(self, model: Model, slots: int, overlap: int = 0):
        self.model = model
        self.slots = slots
        self.h = lib().hso_fast_new(model.h, slots, overlap)

    def __del__(self):
        if getattr(self, "h", None):
            lib().hso_fast_free(self.h)

    def reset(self, slot: int):
        lib().hso_fast_reset(self.h, slot)

    def position(self, slot: int) -> int:
        return lib().hso_fast_position(self.h, slot)

    def run_coded(self, slots, tokens, kinds, values, bits: int = 32, threads: int | None = None,
                  lanes: bool = False) -> np.ndarray:
        """{symbol, start, freq} per input. `lanes`: a decode step (one row per slot) runs in lockstep
        groups of up to 8 slots per thread, as the reference's CPU unfold (unfold.rs:215-246)."""
        s = np.ascontiguousarray(slots, dtype=np.uint32)
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        k = np.ascontiguousarray(kinds, dtype=np.uint32)
        v = np.ascontiguousarray(values, dtype=np.uint64)
        out = np.zeros((s.size, 3), dtype=np.uint64)
        fn = lib().hso_fast_run_lanes if lanes else lib().hso_fast_run
        rc = fn(self.h, _ptr(s), _ptr(t), s.size, _ptr(k), _ptr(v), bits, _ptr(out), None,
                threads or os.cpu_count() or 1)
        if rc:
            raise OracleError(f"fast run failed: {rc}")
        return out

    def run_weights(self, slots, tokens, threads: int | None = None) -> np.ndarray:
        s = np.ascontiguousarray(slots, dtype=np.uint32)
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.zeros((s.size, self.model.vocab), dtype=np.uint64)
        rc = lib().hso_fast_run(self.h, _ptr(s), _ptr(t), s.size, None, None, 32, None, _ptr(out),
                                threads or os.cpu_count() or 1)
        if rc:
            raise OracleError(f"fast run failed: {rc}")
        return out
