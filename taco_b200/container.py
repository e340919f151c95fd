"""The `.taco` container, format versions 1 and 2: parse and build (host side, no GPU).

This mirrors `crates/taco-format` of the reference (the layout table of
crates/taco-format/src/lib.rs:13-35, the header checks of src/header.rs:220-330 and the
parser of src/reader.rs). The backend itself never reads a container; the fold and unfold glue
around it does, and the tests use it to take the coded blocks out of the conformance vectors.

Layout (little-endian): magic "TACO", version u16, flags u16 = 0, model hash [32],
original length u64, checksum SHA-256 [32], block size u32, block count u32; version 2 adds
profile u8, reserved u8, coding parts u16 (bit 0 mixer, bit 1 overlap) and 12 bytes of coding
parameters (byte 0 mixer rule, bytes 2..4 the overlap K). Then the block table (kind u8,
stored length u32 per block) and the stored bytes of every block.
"""

from __future__ import annotations

import ctypes
import ctypes.util
import hashlib
import struct
from dataclasses import dataclass, field

MAGIC = b"TACO"
HEADER_LEN_V1 = 88
HEADER_LEN = 104
MAX_BLOCK_SIZE = 64 * 1024 * 1024
KIND_RAW, KIND_CODED, KIND_ZSTD, KIND_MIXED = 0, 1, 2, 3
KIND_NAMES = {KIND_RAW: "raw", KIND_CODED: "coded", KIND_ZSTD: "zstd", KIND_MIXED: "mixed"}
PROFILE_TEXT, PROFILE_LOGS = 0, 1


class FormatError(ValueError):
    """A container that breaks a rule of the format."""


@dataclass
class Block:
    index: int
    kind: int
    original_len: int
    stored: bytes


@dataclass
class Container:
    version: int
    model_hash: bytes
    original_len: int
    checksum: bytes
    block_size: int
    profile: int = PROFILE_TEXT
    mixer_rule: int = 0
    overlap: int = 0
    blocks: list[Block] = field(default_factory=list)

    @property
    def needs_model(self) -> bool:
        return self.model_hash != bytes(32)


def parse(data: bytes) -> Container:
    """Parses and checks a container (crates/taco-format/src/reader.rs Container::parse)."""
    if len(data) < 6:
        raise FormatError("truncated header")
    if data[:4] != MAGIC:
        raise FormatError("bad magic")
    (version,) = struct.unpack_from("<H", data, 4)
    if version not in (1, 2):
        raise FormatError(f"unsupported version {version}")
    hlen = HEADER_LEN_V1 if version == 1 else HEADER_LEN
    if len(data) < hlen:
        raise FormatError("truncated header")
    (flags,) = struct.unpack_from("<H", data, 6)
    if flags != 0:
        raise FormatError("unknown flags")
    model_hash = data[8:40]
    (original_len,) = struct.unpack_from("<Q", data, 40)
    checksum = data[48:80]
    block_size, block_count = struct.unpack_from("<II", data, 80)
    if block_size == 0 or block_size > MAX_BLOCK_SIZE:
        raise FormatError("block size out of range")
    if block_count != -(-original_len // block_size):
        raise FormatError("wrong block count")
    c = Container(version, model_hash, original_len, checksum, block_size)
    if version == 2:
        profile, reserved, bits = struct.unpack_from("<BBH", data, 88)
        params = data[92:104]
        if profile not in (PROFILE_TEXT, PROFILE_LOGS) or reserved != 0 or bits & ~3:
            raise FormatError("bad version 2 fields")
        if profile == PROFILE_TEXT and bits & 1:
            raise FormatError("the text profile has no mixer")
        if bits & 1:
            if params[0] not in (1, 2):
                raise FormatError("unknown mixer rule")
            c.mixer_rule = params[0]
        elif params[0] != 0:
            raise FormatError("mixer rule without the mixer bit")
        (k,) = struct.unpack_from("<H", params, 2)
        if bits & 2:
            if k == 0:
                raise FormatError("overlap bit with K = 0")
            c.overlap = k
        elif k != 0:
            raise FormatError("overlap without the overlap bit")
        if params[1] != 0 or any(params[4:]):
            raise FormatError("non-zero coding parameters")
        c.profile = profile
    table_end = hlen + 5 * block_count
    if len(data) < table_end:
        raise FormatError("truncated block table")
    off = table_end
    remaining = original_len
    for i in range(block_count):
        kind, stored_len = struct.unpack_from("<BI", data, hlen + 5 * i)
        olen = min(block_size, remaining)
        remaining -= olen
        if kind not in KIND_NAMES or (version == 1 and kind in (KIND_ZSTD, KIND_MIXED)):
            raise FormatError("unknown block kind")
        if kind == KIND_RAW and stored_len != olen:
            raise FormatError("a raw block stores its original bytes")
        if kind != KIND_RAW and stored_len >= olen:
            raise FormatError("a coded, mixed or zstd block is smaller than its original bytes")
        if kind in (KIND_CODED, KIND_MIXED) and not c.needs_model:
            raise FormatError("a coded block needs a model")
        if kind == KIND_MIXED and c.mixer_rule == 0:
            raise FormatError("a mixed block needs the mixer bit")
        if off + stored_len > len(data):
            raise FormatError("truncated block")
        c.blocks.append(Block(i, kind, olen, bytes(data[off:off + stored_len])))
        off += stored_len
    if off != len(data):
        raise FormatError("extra bytes after the last block")
    return c


def build(c: Container) -> bytes:
    """The bytes of a version 2 container (crates/taco-format/src/writer.rs Container::build)."""
    bits = (1 if c.mixer_rule else 0) | (2 if c.overlap else 0)
    params = bytearray(12)
    params[0] = c.mixer_rule
    struct.pack_into("<H", params, 2, c.overlap)
    out = bytearray()
    out += MAGIC + struct.pack("<HH", 2, 0) + c.model_hash + struct.pack("<Q", c.original_len)
    out += c.checksum + struct.pack("<II", c.block_size, len(c.blocks))
    out += struct.pack("<BBH", c.profile, 0, bits) + bytes(params)
    for b in c.blocks:
        out += struct.pack("<BI", b.kind, len(b.stored))
    for b in c.blocks:
        out += b.stored
    return bytes(out)


def sha256(data: bytes) -> bytes:
    return hashlib.sha256(data).digest()


_zstd = None


def decode_zstd(frame: bytes, original_len: int) -> bytes:
    """Decodes a zstd block with the system libzstd (the frame format does not depend on the
    library version). ADR 0011 §5 of the reference: the frame must give exactly the block."""
    global _zstd
    if _zstd is None:
        name = ctypes.util.find_library("zstd") or "libzstd.so.1"
        lib = ctypes.CDLL(name)
        lib.ZSTD_decompress.restype = ctypes.c_size_t
        lib.ZSTD_decompress.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t]
        lib.ZSTD_isError.restype = ctypes.c_uint
        lib.ZSTD_isError.argtypes = [ctypes.c_size_t]
        _zstd = lib
    dst = ctypes.create_string_buffer(max(1, original_len))
    n = _zstd.ZSTD_decompress(dst, original_len, frame, len(frame))
    if _zstd.ZSTD_isError(n) or n != original_len:
        raise FormatError("a zstd block does not decode to its length")
    return dst.raw[:original_len]
