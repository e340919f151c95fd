"""The Python host side of the B200 HardShell backend: the API of the reference's CUDA engine
(crates/hardshell-cuda: CudaDevice, CudaModel, CudaBatch) over the C ABI of
libhardshell_b200.so (include/hardshell_b200.h).

There is no CPU fallback: if the library or a GPU is missing, every call raises.
"""

from __future__ import annotations

import ctypes
import os
import weakref
from dataclasses import dataclass
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libhardshell_b200.so"

HS_OK, HS_NO_DEVICE, HS_CUDA, HS_UNSUPPORTED, HS_MODEL = 0, 1, 2, 3, 4
HS_BAD_SLOT, HS_LENGTH_MISMATCH, HS_TOKEN_RANGE, HS_INVALID_OVERLAP, HS_BAD_ARGUMENT = 5, 6, 7, 8, 9
HS_FORMAT, HS_CORRUPT, HS_MODEL_MISMATCH, HS_IO = 10, 11, 12, 13
_NAMES = {
    HS_NO_DEVICE: "NoDevice", HS_CUDA: "Cuda", HS_UNSUPPORTED: "Unsupported", HS_MODEL: "Model",
    HS_BAD_SLOT: "BadSlot", HS_LENGTH_MISMATCH: "LengthMismatch", HS_TOKEN_RANGE: "TokenOutOfRange",
    HS_INVALID_OVERLAP: "InvalidOverlap", HS_BAD_ARGUMENT: "BadArgument", HS_FORMAT: "Format",
    HS_CORRUPT: "CorruptBlock", HS_MODEL_MISMATCH: "ModelHashMismatch", HS_IO: "Io",
}

ENCODE, DECODE = 0, 1


class HardShellError(RuntimeError):
    """An error of the backend; `code` is the hs_status (crates/hardshell-cuda/src/error.rs)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{_NAMES.get(code, code)}: {message}")
        self.code = code
        self.kind = _NAMES.get(code, str(code))


class Interval(ctypes.Structure):
    _fields_ = [("symbol", ctypes.c_uint32), ("is_last", ctypes.c_uint32), ("start", ctypes.c_uint64),
                ("freq", ctypes.c_uint64), ("reserved", ctypes.c_uint64)]


class ModelInfo(ctypes.Structure):
    _fields_ = [("n_layer", ctypes.c_uint32), ("n_head", ctypes.c_uint32), ("d_model", ctypes.c_uint32),
                ("d_ff", ctypes.c_uint32), ("vocab", ctypes.c_uint32), ("n_ctx", ctypes.c_uint32),
                ("eot_token", ctypes.c_uint32), ("version", ctypes.c_uint32),
                ("cache_bytes_per_slot", ctypes.c_uint64), ("weight_bytes", ctypes.c_uint64),
                ("hash", ctypes.c_uint8 * 32)]


class OpProfile(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("ms", ctypes.c_double), ("launches", ctypes.c_uint64),
                ("ops", ctypes.c_uint64)]


class MixStats(ctypes.Structure):
    """hs_mix_stats (crates/hardshell-cuda/src/mixed.rs:36-47 MixStats)."""
    _fields_ = [("total", ctypes.c_uint64), ("predicted", ctypes.c_uint64), ("top", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32)]


class FoldOptions(ctypes.Structure):
    _fields_ = [("block_size", ctypes.c_uint32), ("overlap", ctypes.c_uint32), ("spread", ctypes.c_uint32),
                ("threads", ctypes.c_uint32)]


class FoldStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("original_len", "container_len", "blocks", "coded_blocks",
                                               "zstd_blocks", "tokens")] + \
               [("block_size", ctypes.c_uint32), ("gpus_failed", ctypes.c_uint32), ("gpu_rows", ctypes.c_uint64),
                ("prep_ms", ctypes.c_double), ("gpu_ms", ctypes.c_double), ("finish_ms", ctypes.c_double)]


SOURCE_FN = ctypes.CFUNCTYPE(ctypes.c_int64, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint8), ctypes.c_size_t)
SINK_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint8),
                           ctypes.c_size_t)
READ_AT_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint8),
                              ctypes.c_size_t)
WRITE_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint8), ctypes.c_size_t)

MIXER_FN = ctypes.CFUNCTYPE(ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(MixStats))
MIX_NONE = 0xFFFFFFFF   # a mixed table without a prediction: the weights max(1, w)
MIX_PLAIN = 0xFFFFFFFE  # the table of GPT-2 alone

INTERVAL_DTYPE = np.dtype([("symbol", "<u4"), ("is_last", "<u4"), ("start", "<u8"), ("freq", "<u8"),
                           ("reserved", "<u8")])

_lib = None


def lib() -> ctypes.CDLL:
    """The backend library. Raises if it is not built (no silent fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise HardShellError(HS_NO_DEVICE, f"{LIB_PATH.name} is not built: run python -m taco_b200.build")
    L = ctypes.CDLL(str(LIB_PATH))
    vp, u32, u64, i32 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
    L.hs_open.argtypes = [i32, ctypes.POINTER(vp)]
    L.hs_dev_free.argtypes = [vp]
    L.hs_dev_free.restype = None
    L.hs_mem_info.argtypes = [vp, ctypes.POINTER(u64), ctypes.POINTER(u64)]
    L.hs_dev_name.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t]
    L.hs_model_load.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(vp)]
    L.hs_model_check.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ModelInfo)]
    L.hs_model_free.argtypes = [vp]
    L.hs_model_free.restype = None
    L.hs_model_get_info.argtypes = [vp, ctypes.POINTER(ModelInfo)]
    L.hs_batch_new.argtypes = [vp, u32, u32, ctypes.POINTER(vp)]
    L.hs_batch_free.argtypes = [vp]
    L.hs_batch_free.restype = None
    L.hs_batch_set_overlap.argtypes = [vp, ctypes.c_uint16]
    L.hs_batch_reset.argtypes = [vp, u32]
    L.hs_batch_position.argtypes = [vp, u32]
    L.hs_batch_position.restype = u32
    L.hs_batch_gpu_bytes.argtypes = [vp]
    L.hs_batch_gpu_bytes.restype = u64
    L.hs_batch_run_coded.argtypes = [vp, vp, vp, vp, vp, u32, u32, vp]
    L.hs_batch_run_weights.argtypes = [vp, vp, vp, u32, vp]
    L.hs_batch_run_coded_mixed.argtypes = [vp, vp, vp, vp, vp, vp, u32, u32, MIXER_FN, vp, vp]
    L.hs_batch_run_coded_dual.argtypes = [vp, vp, vp, vp, vp, u32, u32, MIXER_FN, vp, vp, vp]
    L.hs_batch_stream_len.argtypes = [vp, u32, ctypes.POINTER(ctypes.c_uint64)]
    L.hs_batch_room.argtypes = [vp, u32, ctypes.POINTER(ctypes.c_uint64)]
    L.hs_batch_truncate.argtypes = [vp, u32, ctypes.c_uint64]
    L.hs_batch_decode_blocks.argtypes = [vp, u32, vp, vp, ctypes.c_uint64, vp, vp, vp, u32, vp, ctypes.c_uint64, vp, vp]
    L.hs_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    L.hs_tokenizer_new.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(vp)]
    L.hs_tokenizer_free.argtypes = [vp]
    L.hs_tokenizer_free.restype = None
    L.hs_tokenize.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t, vp, ctypes.c_size_t,
                              ctypes.POINTER(ctypes.c_size_t)]
    L.hs_tokenizer_pieces.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t, vp, ctypes.c_size_t,
                                      ctypes.POINTER(ctypes.c_size_t)]
    L.hs_fold_bound.argtypes = [u64, u32]
    L.hs_fold_bound.restype = u64
    L.hs_fold.argtypes = [vp, vp, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(FoldOptions), vp, ctypes.c_size_t,
                          ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(FoldStats)]
    L.hs_fold_multi.argtypes = [vp, u32, ctypes.c_char_p, ctypes.c_size_t, u32, u32, vp, ctypes.c_char_p,
                                ctypes.c_size_t, ctypes.POINTER(FoldOptions), vp, ctypes.c_size_t,
                                ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(FoldStats)]
    L.hs_unfold.argtypes = [vp, vp, ctypes.c_char_p, ctypes.c_size_t, vp, ctypes.c_size_t,
                            ctypes.POINTER(ctypes.c_size_t)]
    L.hs_fold_stream.argtypes = [vp, vp, u64, SOURCE_FN, vp, SINK_FN, vp, ctypes.POINTER(FoldOptions),
                                 ctypes.POINTER(u64), ctypes.POINTER(FoldStats)]
    L.hs_fold_stream_multi.argtypes = [vp, u32, ctypes.c_char_p, ctypes.c_size_t, u32, u32, vp, u64, SOURCE_FN, vp,
                                       SINK_FN, vp, ctypes.POINTER(FoldOptions), ctypes.POINTER(u64),
                                       ctypes.POINTER(FoldStats)]
    L.hs_unfold_multi.argtypes = [vp, u32, ctypes.c_char_p, ctypes.c_size_t, u32, u32, vp, ctypes.c_char_p,
                                  ctypes.c_size_t, vp, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]
    L.hs_unfold_stream.argtypes = [vp, vp, u64, READ_AT_FN, vp, WRITE_FN, vp, ctypes.POINTER(u64)]
    L.hs_fold_spool.argtypes = [vp, vp, u64, SOURCE_FN, vp, WRITE_FN, vp, ctypes.c_char_p,
                                ctypes.POINTER(FoldOptions), ctypes.POINTER(u64), ctypes.POINTER(FoldStats)]
    L.hs_fold_spool_multi.argtypes = [vp, u32, ctypes.c_char_p, ctypes.c_size_t, u32, u32, vp, u64, SOURCE_FN, vp,
                                      WRITE_FN, vp, ctypes.c_char_p, ctypes.POINTER(FoldOptions),
                                      ctypes.POINTER(u64), ctypes.POINTER(FoldStats)]
    L.hs_unfold_stream_multi.argtypes = [vp, u32, ctypes.c_char_p, ctypes.c_size_t, u32, u32, vp, u64, READ_AT_FN,
                                         vp, WRITE_FN, vp, ctypes.POINTER(u64)]
    L.hs_unfold_pipe.argtypes = [vp, vp, SOURCE_FN, vp, WRITE_FN, vp, ctypes.POINTER(u64)]
    L.hs_unfold_pipe_multi.argtypes = [vp, u32, ctypes.c_char_p, ctypes.c_size_t, u32, u32, vp, SOURCE_FN, vp,
                                       WRITE_FN, vp, ctypes.POINTER(u64)]
    L.hs_zstd_version.argtypes = []
    L.hs_zstd_version.restype = u32
    L.hs_op_linear_act.argtypes = [vp, i32, vp, vp, vp, vp, u32, u32, u32, u32, vp, vp]
    L.hs_op_linear_act_noalloc.argtypes = [vp, i32, vp, vp, vp, vp, u32, u32, u32, u32, vp, vp]
    L.hs_op_linear_bench.argtypes = [vp, i32, u32, u32, u32, u64, i32, i32, ctypes.POINTER(ctypes.c_double)]
    L.hs_batch_set_profiling.argtypes = [vp, i32]
    L.hs_batch_profile.argtypes = [vp, vp, i32]
    L.hs_launch_count.argtypes = []
    L.hs_launch_count.restype = u64
    _lib = L
    return L


def _check(rc: int):
    if rc != HS_OK:
        buf = ctypes.create_string_buffer(1024)
        lib().hs_last_error(buf, 1024)
        raise HardShellError(rc, buf.value.decode(errors="replace"))


def _p(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


def launch_count() -> int:
    """Kernel launches of the library in this process."""
    return int(lib().hs_launch_count())


class Tokenizer:
    """crates/taco/src/tokenizer Tokenizer: GPT-2 byte-level BPE of a .hsm model (host code, no GPU)."""

    def __init__(self, model_file: bytes):
        h = ctypes.c_void_p()
        _check(lib().hs_tokenizer_new(model_file, len(model_file), ctypes.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().hs_tokenizer_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def encode(self, data: bytes) -> np.ndarray:
        out = np.zeros(max(len(data), 1), dtype=np.uint32)
        n = ctypes.c_size_t()
        _check(lib().hs_tokenize(self.h, data, len(data), _p(out), out.size, ctypes.byref(n)))
        return out[:n.value].copy()

    def pieces(self, data: bytes) -> list[bytes]:
        """The pre-tokenizer's pieces of `data` (and the single bytes outside UTF-8 runs)."""
        ends = np.zeros(max(len(data), 1), dtype=np.uint64)
        n = ctypes.c_size_t()
        _check(lib().hs_tokenizer_pieces(self.h, data, len(data), _p(ends), ends.size, ctypes.byref(n)))
        out, a = [], 0
        for e in ends[:n.value].tolist():
            out.append(data[a:e])
            a = e
        return out


def check_model(data: bytes) -> dict:
    """hs_model_check: the host-side validation of a .hsm file (Model::load without a device); its
    dimensions and SHA-256, or HardShellError(HS_MODEL)."""
    info = ModelInfo()
    _check(lib().hs_model_check(data, len(data), ctypes.byref(info)))
    out = {name: getattr(info, name) for name, _ in ModelInfo._fields_ if name != "hash"}
    out["hash"] = bytes(info.hash)
    return out


def fold(batch, tokenizer, data: bytes, block_size: int = 0, overlap: int = 0, spread: bool = False,
         threads: int = 0):
    """taco::fold_with on the CUDA engine, profile text (hs_fold): (container bytes, stats dict)."""
    opt = FoldOptions(block_size, overlap, int(spread), threads)
    cap = int(lib().hs_fold_bound(len(data), block_size))
    out = np.zeros(max(cap, 1), dtype=np.uint8)
    n = ctypes.c_size_t()
    st = FoldStats()
    _check(lib().hs_fold(batch.h, tokenizer.h, data, len(data), ctypes.byref(opt), _p(out), out.size,
                         ctypes.byref(n), ctypes.byref(st)))
    stats = {name: getattr(st, name) for name, _ in FoldStats._fields_}
    return out[:n.value].tobytes(), stats


def fold_multi(ordinals, model_file: bytes, tokenizer, data: bytes, block_size: int = 0, overlap: int = 0,
               slots: int = 256, max_rows: int = 16384, spread: bool = False, threads: int = 0):
    """hs_fold_multi: the fold of `data` on the GPUs `ordinals`, one host thread each."""
    ords = np.ascontiguousarray(ordinals, dtype=np.int32)
    opt = FoldOptions(block_size, overlap, int(spread), threads)
    cap = int(lib().hs_fold_bound(len(data), block_size))
    out = np.zeros(max(cap, 1), dtype=np.uint8)
    n = ctypes.c_size_t()
    st = FoldStats()
    _check(lib().hs_fold_multi(_p(ords), ords.size, model_file, len(model_file), slots, max_rows, tokenizer.h, data,
                               len(data), ctypes.byref(opt), _p(out), out.size, ctypes.byref(n), ctypes.byref(st)))
    stats = {name: getattr(st, name) for name, _ in FoldStats._fields_}
    return out[:n.value].tobytes(), stats


def _source(read):
    """A ctypes source over read(n) -> bytes (at most n; b"" at the end). An exception, or more
    than n bytes, fails the call with HS_IO."""

    def source(_user, buf, cap):
        try:
            data = read(cap)
        except Exception:  # noqa: BLE001 - any failure of the caller's source is an I/O error
            return -1
        if len(data) > cap:
            return -1
        ctypes.memmove(buf, data, len(data))
        return len(data)

    return SOURCE_FN(source)


def _writer(write):
    """A ctypes in-order writer over write(data). An exception fails the call with HS_IO."""

    def wr(_user, buf, n):
        try:
            write(ctypes.string_at(buf, n))
        except Exception:  # noqa: BLE001
            return 1
        return 0

    return WRITE_FN(wr)


def _stream_callbacks(read, write):
    """ctypes callbacks over Python file-like callables: read(n) -> bytes (the source),
    write(at, data) (the seekable sink). An exception in either fails the call with HS_IO."""

    def sink(_user, at, buf, n):
        try:
            write(at, ctypes.string_at(buf, n))
        except Exception:  # noqa: BLE001
            return 1
        return 0

    return _source(read), SINK_FN(sink)


def fold_stream(batch, tokenizer, length: int, read, write, block_size: int = 0, overlap: int = 0,
                spread: bool = False, threads: int = 0):
    """hs_fold_stream: the fold of the `length` bytes that read(n) gives, into the seekable sink
    write(at, data); returns (container length, stats)."""
    opt = FoldOptions(block_size, overlap, int(spread), threads)
    src, snk = _stream_callbacks(read, write)
    n = ctypes.c_uint64()
    st = FoldStats()
    _check(lib().hs_fold_stream(batch.h, tokenizer.h, length, src, None, snk, None, ctypes.byref(opt), ctypes.byref(n),
                                ctypes.byref(st)))
    return n.value, {name: getattr(st, name) for name, _ in FoldStats._fields_}


def fold_stream_multi(ordinals, model_file: bytes, tokenizer, length: int, read, write, block_size: int = 0,
                      overlap: int = 0, slots: int = 256, max_rows: int = 16384, spread: bool = False,
                      threads: int = 0):
    """hs_fold_stream_multi: fold_stream on the GPUs `ordinals`, one host thread each."""
    ords = np.ascontiguousarray(ordinals, dtype=np.int32)
    opt = FoldOptions(block_size, overlap, int(spread), threads)
    src, snk = _stream_callbacks(read, write)
    n = ctypes.c_uint64()
    st = FoldStats()
    _check(lib().hs_fold_stream_multi(_p(ords), ords.size, model_file, len(model_file), slots, max_rows, tokenizer.h,
                                      length, src, None, snk, None, ctypes.byref(opt), ctypes.byref(n),
                                      ctypes.byref(st)))
    return n.value, {name: getattr(st, name) for name, _ in FoldStats._fields_}


LEN_UNKNOWN = 0xFFFFFFFFFFFFFFFF  # HS_LEN_UNKNOWN: a fold input whose length is known only at its end


def _spool_dir(spool_dir) -> bytes | None:
    return None if spool_dir is None else os.fsencode(spool_dir)


def fold_spool(batch, tokenizer, read, write, length: int | None = None, spool_dir=None, block_size: int = 0,
               overlap: int = 0, spread: bool = False, threads: int = 0):
    """hs_fold_spool (StreamFold::to_writer): the fold of the bytes that read(n) gives (`length`
    of them, or None if it is not known) into the in-order writer write(data), spooling the
    blocks and the table in `spool_dir`; returns (container length, stats)."""
    opt = FoldOptions(block_size, overlap, int(spread), threads)
    src, wr = _source(read), _writer(write)
    n = ctypes.c_uint64()
    st = FoldStats()
    _check(lib().hs_fold_spool(batch.h, tokenizer.h, LEN_UNKNOWN if length is None else length, src, None, wr, None,
                               _spool_dir(spool_dir), ctypes.byref(opt), ctypes.byref(n), ctypes.byref(st)))
    return n.value, {name: getattr(st, name) for name, _ in FoldStats._fields_}


def fold_spool_multi(ordinals, model_file: bytes, tokenizer, read, write, length: int | None = None, spool_dir=None,
                     block_size: int = 0, overlap: int = 0, slots: int = 256, max_rows: int = 16384,
                     spread: bool = False, threads: int = 0):
    """hs_fold_spool_multi: fold_spool on the GPUs `ordinals`, one host thread each (a fold whose
    blocks need no model window opens no GPU)."""
    ords = np.ascontiguousarray(ordinals, dtype=np.int32)
    opt = FoldOptions(block_size, overlap, int(spread), threads)
    src, wr = _source(read), _writer(write)
    n = ctypes.c_uint64()
    st = FoldStats()
    _check(lib().hs_fold_spool_multi(_p(ords), ords.size, model_file, len(model_file), slots, max_rows, tokenizer.h,
                                     LEN_UNKNOWN if length is None else length, src, None, wr, None,
                                     _spool_dir(spool_dir), ctypes.byref(opt), ctypes.byref(n), ctypes.byref(st)))
    return n.value, {name: getattr(st, name) for name, _ in FoldStats._fields_}


def unfold_pipe(batch, tokenizer, read, write) -> int:
    """hs_unfold_pipe (StreamUnfold::from_reader): the unfold of the container that read(n)
    gives in one pass, into write(data); returns the original length."""
    src, wr = _source(read), _writer(write)
    n = ctypes.c_uint64()
    _check(lib().hs_unfold_pipe(batch.h, tokenizer.h, src, None, wr, None, ctypes.byref(n)))
    return n.value


def unfold_pipe_multi(ordinals, model_file: bytes, tokenizer, read, write, slots: int = 256,
                      max_rows: int = 16384) -> int:
    """hs_unfold_pipe_multi: unfold_pipe with the worker threads of unfold_multi (a container
    without coded blocks opens no GPU); returns the original length."""
    ords = np.ascontiguousarray(ordinals, dtype=np.int32)
    src, wr = _source(read), _writer(write)
    n = ctypes.c_uint64()
    _check(lib().hs_unfold_pipe_multi(_p(ords), ords.size, model_file, len(model_file), slots, max_rows, tokenizer.h,
                                      src, None, wr, None, ctypes.byref(n)))
    return n.value


def _read_at(read_at):
    """A ctypes positional reader over read_at(at, n) -> bytes (exactly n). An exception or a
    short read fails the read."""

    def ra(_user, at, buf, n):
        try:
            data = read_at(at, n)
        except Exception:  # noqa: BLE001
            return 1
        if len(data) != n:
            return 1
        ctypes.memmove(buf, data, n)
        return 0

    return READ_AT_FN(ra)


def unfold_stream(batch, tokenizer, length: int, read_at, write) -> int:
    """hs_unfold_stream: the unfold of the `length`-byte container that read_at(at, n) -> bytes
    reads, into write(data); returns the original length."""
    cb_ra, cb_wr = _read_at(read_at), _writer(write)
    n = ctypes.c_uint64()
    _check(lib().hs_unfold_stream(batch.h, tokenizer.h, length, cb_ra, None, cb_wr, None, ctypes.byref(n)))
    return n.value


def unfold_stream_multi(ordinals, model_file: bytes, tokenizer, length: int, read_at, write, slots: int = 256,
                        max_rows: int = 16384) -> int:
    """hs_unfold_stream_multi: unfold_stream with the worker threads of unfold_multi (a container
    without coded blocks opens no GPU); returns the original length."""
    ords = np.ascontiguousarray(ordinals, dtype=np.int32)
    cb_ra, cb_wr = _read_at(read_at), _writer(write)
    n = ctypes.c_uint64()
    _check(lib().hs_unfold_stream_multi(_p(ords), ords.size, model_file, len(model_file), slots, max_rows,
                                        tokenizer.h, length, cb_ra, None, cb_wr, None, ctypes.byref(n)))
    return n.value


def unfold_multi(ordinals, model_file: bytes, tokenizer, container: bytes, slots: int = 256,
                 max_rows: int = 16384) -> bytes:
    """hs_unfold_multi: the unfold of a .taco container with its coded blocks dealt to worker
    threads on the GPUs `ordinals`."""
    ords = np.ascontiguousarray(ordinals, dtype=np.int32)
    original_len = int.from_bytes(container[40:48], "little") if len(container) >= 48 else 0
    out = np.zeros(max(original_len, 1), dtype=np.uint8)
    n = ctypes.c_size_t()
    _check(lib().hs_unfold_multi(_p(ords), ords.size, model_file, len(model_file), slots, max_rows, tokenizer.h,
                                 container, len(container), _p(out), out.size, ctypes.byref(n)))
    return out[:n.value].tobytes()


def unfold(batch, tokenizer, container: bytes, original_len: int | None = None) -> bytes:
    """taco::unfold on the CUDA engine (hs_unfold): the original bytes of a .taco container."""
    if original_len is None:
        original_len = int.from_bytes(container[40:48], "little") if len(container) >= 48 else 0
    out = np.zeros(max(original_len, 1), dtype=np.uint8)
    n = ctypes.c_size_t()
    _check(lib().hs_unfold(batch.h, tokenizer.h, container, len(container), _p(out), out.size, ctypes.byref(n)))
    return out[:n.value].tobytes()


def zstd_version() -> int:
    return int(lib().hs_zstd_version())


class CudaDevice:
    """crates/hardshell-cuda/src/device.rs CudaDevice: one GPU (use it on one thread)."""

    def __init__(self, ordinal: int = 0):
        h = ctypes.c_void_p()
        _check(lib().hs_open(ordinal, ctypes.byref(h)))
        self.h = h
        self.ordinal = ordinal
        self._children = weakref.WeakSet()  # the models loaded on this device

    def close(self):
        """Frees the device after its models (and their batches), the order in which the
        reference's borrows end (a model borrows its device, a batch its model)."""
        if getattr(self, "h", None):
            for c in list(self._children):
                c.close()
            lib().hs_dev_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    @property
    def name(self) -> str:
        buf = ctypes.create_string_buffer(256)
        _check(lib().hs_dev_name(self.h, buf, 256))
        return buf.value.decode()

    def memory(self) -> tuple[int, int]:
        f, t = ctypes.c_uint64(), ctypes.c_uint64()
        _check(lib().hs_mem_info(self.h, ctypes.byref(f), ctypes.byref(t)))
        return f.value, t.value

    def linear_act(self, A: np.ndarray, W: np.ndarray, bias: np.ndarray, mult: np.ndarray, shift: int,
                   path: str = "tc") -> np.ndarray:
        """The linear op alone: clamp(rescale(A . W^T + b, m, s), -127, 127) (tests)."""
        A = np.ascontiguousarray(A, dtype=np.int8)
        W = np.ascontiguousarray(W, dtype=np.int8)
        b = np.ascontiguousarray(bias, dtype=np.int32)
        m = np.ascontiguousarray(mult, dtype=np.int32)
        M, K = A.shape
        N = W.shape[0]
        out = np.zeros((M, N), dtype=np.int8)
        _check(lib().hs_op_linear_act(self.h, 0 if path == "tc" else 1, _p(A), _p(W), _p(b), _p(m), shift, M, N, K,
                                      _p(out), None))
        return out

    def matmul_raw(self, A: np.ndarray, W: np.ndarray, path: str = "tc") -> np.ndarray:
        """The exact int32 accumulators A . W^T (tests)."""
        A = np.ascontiguousarray(A, dtype=np.int8)
        W = np.ascontiguousarray(W, dtype=np.int8)
        M, K = A.shape
        N = W.shape[0]
        out = np.zeros((M, N), dtype=np.int32)
        _check(lib().hs_op_linear_act(self.h, 0 if path == "tc" else 1, _p(A), _p(W), None, None, 0, M, N, K, None,
                                      _p(out)))
        return out

    def linear_act_noalloc(self, A: np.ndarray, W: np.ndarray, bias: np.ndarray | None, mult: np.ndarray | None,
                           shift: int, path: str = "tc", raw: bool = False) -> np.ndarray:
        """linear_act (or matmul_raw with raw=True) through the entry point that stages everything in
        the library's static device array instead of allocating (HS_STATIC_SCRATCH_BYTES)."""
        A = np.ascontiguousarray(A, dtype=np.int8)
        W = np.ascontiguousarray(W, dtype=np.int8)
        M, K = A.shape
        N = W.shape[0]
        if raw:
            out = np.zeros((M, N), dtype=np.int32)
            _check(lib().hs_op_linear_act_noalloc(self.h, 0 if path == "tc" else 1, _p(A), _p(W), None, None, 0,
                                                  M, N, K, None, _p(out)))
            return out
        b = np.ascontiguousarray(bias, dtype=np.int32)
        m = np.ascontiguousarray(mult, dtype=np.int32)
        out = np.zeros((M, N), dtype=np.int8)
        _check(lib().hs_op_linear_act_noalloc(self.h, 0 if path == "tc" else 1, _p(A), _p(W), _p(b), _p(m), shift,
                                              M, N, K, _p(out), None))
        return out

    def linear_bench(self, M: int, N: int, K: int, seed: int = 1, warmup: int = 3, iters: int = 20,
                     path: str = "tc") -> float:
        """Mean microseconds of one device-resident linear launch (bench.py)."""
        us = ctypes.c_double()
        _check(lib().hs_op_linear_bench(self.h, 0 if path == "tc" else 1, M, N, K, seed, warmup, iters,
                                        ctypes.byref(us)))
        return us.value


@dataclass
class Info:
    n_layer: int
    n_head: int
    d_model: int
    d_ff: int
    vocab: int
    n_ctx: int
    eot_token: int
    version: int
    cache_bytes_per_slot: int
    weight_bytes: int
    hash: bytes


class CudaModel:
    """crates/hardshell-cuda/src/model.rs CudaModel: a validated .hsm model on one device."""

    def __init__(self, device: CudaDevice, data: bytes):
        if not device.h:
            raise HardShellError(HS_BAD_ARGUMENT, "the device is closed")
        self.device = device
        h = ctypes.c_void_p()
        _check(lib().hs_model_load(device.h, bytes(data), len(data), ctypes.byref(h)))
        self.h = h
        self._children = weakref.WeakSet()  # the batches of this model
        device._children.add(self)
        mi = ModelInfo()
        _check(lib().hs_model_get_info(self.h, ctypes.byref(mi)))
        self.info = Info(mi.n_layer, mi.n_head, mi.d_model, mi.d_ff, mi.vocab, mi.n_ctx, mi.eot_token, mi.version,
                         mi.cache_bytes_per_slot, mi.weight_bytes, bytes(mi.hash))

    def close(self):
        if getattr(self, "h", None):
            for c in list(self._children):
                c.close()
            lib().hs_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def vocab_size(self) -> int:
        return self.info.vocab

    def n_ctx(self) -> int:
        return self.info.n_ctx

    def eot_token(self) -> int:
        return self.info.eot_token

    def hash(self) -> bytes:
        return self.info.hash

    def cache_bytes_per_slot(self) -> int:
        return self.info.cache_bytes_per_slot


class CudaBatch:
    """crates/hardshell-cuda/src/batch.rs CudaBatch: `slots` sessions that run together."""

    def __init__(self, model: CudaModel, slots: int, max_rows: int):
        if not model.h:
            raise HardShellError(HS_BAD_ARGUMENT, "the model is closed")
        self.model = model
        h = ctypes.c_void_p()
        _check(lib().hs_batch_new(model.h, slots, max_rows, ctypes.byref(h)))
        self.h = h
        model._children.add(self)
        self.slots = slots
        self.max_rows = max(2, max_rows)

    def close(self):
        if getattr(self, "h", None):
            lib().hs_batch_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def set_overlap(self, k: int):
        _check(lib().hs_batch_set_overlap(self.h, k))

    def reset(self, slot: int):
        _check(lib().hs_batch_reset(self.h, slot))

    def position(self, slot: int) -> int:
        return lib().hs_batch_position(self.h, slot)

    def gpu_bytes(self) -> int:
        return lib().hs_batch_gpu_bytes(self.h)

    def set_profiling(self, on: bool):
        """CudaBatch::profile: per-op device time from CUDA events around each launch."""
        _check(lib().hs_batch_set_profiling(self.h, int(on)))

    def profile(self) -> dict[str, dict]:
        arr = (OpProfile * 32)()
        n = lib().hs_batch_profile(self.h, arr, 32)
        if n < 0:
            _check(n)
        return {arr[i].name.decode(): {"ms": arr[i].ms, "launches": arr[i].launches, "ops": arr[i].ops}
                for i in range(n)}

    def run_coded(self, slots, tokens, kinds, values, freq_bits: int = 32, out: np.ndarray | None = None) -> np.ndarray:
        """The coder answers of the inputs: a structured array (symbol, is_last, start, freq).
        `out`, if given, is a caller-owned INTERVAL_DTYPE array of the inputs' length that receives
        the answers (a caller that codes many batches reuses one buffer)."""
        s = np.ascontiguousarray(slots, dtype=np.uint32)
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        k = np.ascontiguousarray(kinds, dtype=np.uint32)
        v = np.ascontiguousarray(values, dtype=np.uint64)
        n = s.size
        if not (t.size == k.size == v.size == n):
            raise HardShellError(HS_LENGTH_MISMATCH, "the inputs and the queries differ in length")
        if out is None:
            out = np.zeros(n, dtype=INTERVAL_DTYPE)
        elif out.dtype != INTERVAL_DTYPE or out.size != n or not out.flags["C_CONTIGUOUS"] or not out.flags["WRITEABLE"]:
            raise HardShellError(HS_LENGTH_MISMATCH, "out must be a writable contiguous interval array of the inputs' length")
        _check(lib().hs_batch_run_coded(self.h, _p(s), _p(t), _p(k), _p(v), n, freq_bits, _p(out)))
        return out

    @staticmethod
    def _mixer(mixer, caught: list):
        """The C callback of a Python mixer(input, total, predicted, top) -> q. An exception in the
        mixer gives q = 0, which fails the call; the caller raises it again."""

        def fn(_user, i, st):
            try:
                return int(mixer(int(i), int(st[0].total), int(st[0].predicted), int(st[0].top)))
            except BaseException as e:  # noqa: BLE001 - re-raised by the caller
                caught.append(e)
                return 0

        return MIXER_FN(fn)

    def run_coded_mixed(self, slots, tokens, kinds, values, tables, freq_bits: int, mixer) -> np.ndarray:
        """CudaBatch::run_coded_mixed: the answers in the table that tables[i] names (a predicted
        token, MIX_NONE or MIX_PLAIN). mixer(input, total, predicted, top) gives q for each input
        with a predicted token, in input order."""
        s = np.ascontiguousarray(slots, dtype=np.uint32)
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        k = np.ascontiguousarray(kinds, dtype=np.uint32)
        v = np.ascontiguousarray(values, dtype=np.uint64)
        tb = np.ascontiguousarray(tables, dtype=np.uint32)
        n = s.size
        if not (t.size == k.size == v.size == tb.size == n):
            raise HardShellError(HS_LENGTH_MISMATCH, "the inputs, queries and tables differ in length")
        out = np.zeros(n, dtype=INTERVAL_DTYPE)
        caught: list = []
        cb = self._mixer(mixer, caught)
        rc = lib().hs_batch_run_coded_mixed(self.h, _p(s), _p(t), _p(k), _p(v), _p(tb), n, freq_bits, cb, None,
                                            _p(out))
        if caught:
            raise caught[0]
        _check(rc)
        return out

    def run_coded_dual(self, slots, tokens, coded, predictions, freq_bits: int, mixer):
        """CudaBatch::run_coded_dual: (intervals of coded[i] in the table of GPT-2 alone, in the mixed
        table of predictions[i]); a prediction is a token or MIX_NONE."""
        s = np.ascontiguousarray(slots, dtype=np.uint32)
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        c = np.ascontiguousarray(coded, dtype=np.uint32)
        pr = np.ascontiguousarray(predictions, dtype=np.uint32)
        n = s.size
        if not (t.size == c.size == pr.size == n):
            raise HardShellError(HS_LENGTH_MISMATCH, "the inputs, tokens and predictions differ in length")
        plain = np.zeros(n, dtype=INTERVAL_DTYPE)
        mixed = np.zeros(n, dtype=INTERVAL_DTYPE)
        caught: list = []
        cb = self._mixer(mixer, caught)
        rc = lib().hs_batch_run_coded_dual(self.h, _p(s), _p(t), _p(c), _p(pr), n, freq_bits, cb, None, _p(plain),
                                           _p(mixed))
        if caught:
            raise caught[0]
        _check(rc)
        return plain, mixed

    def run_weights(self, slots, tokens) -> np.ndarray:
        s = np.ascontiguousarray(slots, dtype=np.uint32)
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        if s.size != t.size:
            raise HardShellError(HS_LENGTH_MISMATCH, "slots and tokens differ in length")
        out = np.zeros((s.size, self.model.info.vocab), dtype=np.uint64)
        _check(lib().hs_batch_run_weights(self.h, _p(s), _p(t), s.size, _p(out)))
        return out

    def stream_len(self, slot: int) -> int:
        """CudaBatch::stream_len: the inputs of `slot` since its last reset."""
        v = ctypes.c_uint64()
        _check(lib().hs_batch_stream_len(self.h, slot, ctypes.byref(v)))
        return v.value

    def room(self, slot: int) -> int:
        """CudaBatch::room: the inputs `slot` can take before its next context restart."""
        v = ctypes.c_uint64()
        _check(lib().hs_batch_room(self.h, slot, ctypes.byref(v)))
        return v.value

    def truncate(self, slot: int, length: int):
        """CudaBatch::truncate: keep the first `length` inputs of `slot`."""
        _check(lib().hs_batch_truncate(self.h, slot, length))

    def decode_blocks(self, slots, payloads, counts, freq_bits: int = 32):
        """hs_batch_decode_blocks: block i (the range-coded bytes payloads[i], counts[i] tokens) is
        decoded in slot slots[i] with the decoder on the device. Returns (tokens per block, status
        per block: 0, or 1 if an interval did not hold its target)."""
        s = np.ascontiguousarray(slots, dtype=np.uint32)
        cnt = np.ascontiguousarray(counts, dtype=np.uint32)
        n = s.size
        if len(payloads) != n or cnt.size != n:
            raise HardShellError(HS_LENGTH_MISMATCH, "slots, payloads and counts differ in length")
        lens = np.array([len(p) for p in payloads], dtype=np.uint64)
        offs = np.zeros(n, dtype=np.uint64)
        if n:
            offs[1:] = np.cumsum(lens)[:-1]
        buf = np.frombuffer(b"".join(bytes(p) for p in payloads) or b"\0", dtype=np.uint8).copy()
        toff = np.zeros(n, dtype=np.uint64)
        if n:
            toff[1:] = np.cumsum(cnt.astype(np.uint64))[:-1]
        total = int(cnt.astype(np.uint64).sum())
        out = np.zeros(max(total, 1), dtype=np.uint32)
        status = np.zeros(max(n, 1), dtype=np.uint32)
        _check(lib().hs_batch_decode_blocks(self.h, n, _p(s), _p(buf), int(lens.sum()), _p(offs), _p(lens), _p(cnt),
                                            freq_bits, _p(out), total, _p(toff), _p(status)))
        toks = [out[int(toff[i]):int(toff[i]) + int(cnt[i])].copy() for i in range(n)]
        return toks, status[:n].copy()
