"""GGUF container restatement -- TEST INFRASTRUCTURE ONLY.

Pure-Python restatement of the reference's GGUF header parser
(src/gguf_loader.rs:341-408, reader 171-330) and of its in-test GGUF writer
build_gguf_bytes (src/gguf_loader.rs:766-824). Used by tests to check the
product's native GGUF reader; never imported by vortex_b200.
"""
from __future__ import annotations

import struct

GGUF_MAGIC = 0x46475547
GGUF_DEFAULT_ALIGNMENT = 32

# GGUFValueType (src/gguf_loader.rs:21-36)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)

# GGMLQuantType block geometry (src/gguf_loader.rs:61-128): type -> (bytes, elements)
GGML_TYPES = {0: (4, 1), 1: (2, 1), 2: (18, 32), 3: (20, 32), 6: (22, 32), 7: (24, 32),
              8: (34, 32), 10: (84, 256), 11: (110, 256), 12: (144, 256), 13: (176, 256),
              14: (210, 256)}


class GGUFError(Exception):
    pass


class _Reader:
    def __init__(self, data: bytes):
        self.data = data
        self.pos = 0

    def _take(self, n, what):
        if len(self.data) - self.pos < n:
            raise GGUFError(f"unexpected EOF reading {what}")
        b = self.data[self.pos:self.pos + n]
        self.pos += n
        return b

    def u8(self):
        return self._take(1, "u8")[0]

    def u16(self):
        return struct.unpack("<H", self._take(2, "u16"))[0]

    def u32(self):
        return struct.unpack("<I", self._take(4, "u32"))[0]

    def u64(self):
        return struct.unpack("<Q", self._take(8, "u64"))[0]

    def string(self):
        n = self.u64()
        if len(self.data) - self.pos < n:
            raise GGUFError(f"unexpected EOF reading string of length {n}")
        s = self.data[self.pos:self.pos + n]
        self.pos += n
        try:
            return s.decode("utf-8")
        except UnicodeDecodeError as e:
            raise GGUFError(f"invalid UTF-8 in GGUF string: {e}")

    def value(self, t):
        if t == U8:
            return self.u8()
        if t == I8:
            return struct.unpack("<b", bytes([self.u8()]))[0]
        if t == U16:
            return self.u16()
        if t == I16:
            return struct.unpack("<h", struct.pack("<H", self.u16()))[0]
        if t == U32:
            return self.u32()
        if t == I32:
            return struct.unpack("<i", struct.pack("<I", self.u32()))[0]
        if t == F32:
            return struct.unpack("<f", struct.pack("<I", self.u32()))[0]
        if t == BOOL:
            return self.u8() != 0
        if t == STRING:
            return self.string()
        if t == ARRAY:
            et = self.u32()
            if et > 12:
                raise GGUFError(f"unknown GGUF value type: {et}")
            n = self.u64()
            return [self.value(et) for _ in range(n)]
        if t == U64:
            return self.u64()
        if t == I64:
            return struct.unpack("<q", struct.pack("<Q", self.u64()))[0]
        if t == F64:
            return struct.unpack("<d", struct.pack("<Q", self.u64()))[0]
        raise GGUFError(f"unknown GGUF value type: {t}")


def parse_gguf(data: bytes) -> dict:
    """parse_gguf (src/gguf_loader.rs:341-408)."""
    r = _Reader(data)
    magic = r.u32()
    if magic != GGUF_MAGIC:
        raise GGUFError(f"invalid GGUF magic: 0x{magic:08X} (expected 0x{GGUF_MAGIC:08X})")
    version = r.u32()
    if version not in (2, 3):
        raise GGUFError(f"unsupported GGUF version: {version}")
    n_tensors = r.u64()
    n_kv = r.u64()
    meta = {}
    for _ in range(n_kv):
        key = r.string()
        t = r.u32()
        if t > 12:
            raise GGUFError(f"unknown GGUF value type: {t}")
        meta[key] = (t, r.value(t))
    al = meta.get("general.alignment")
    alignment = al[1] if al is not None and al[0] in (U32, U64, I32) else GGUF_DEFAULT_ALIGNMENT
    tensors = []
    for _ in range(n_tensors):
        name = r.string()
        nd = r.u32()
        dims = [r.u64() for _ in range(nd)]
        qt = r.u32()
        if qt not in GGML_TYPES:
            raise GGUFError(f"unknown GGML quant type: {qt}")
        off = r.u64()
        tensors.append({"name": name, "dims": dims, "type": qt, "offset": off})
    data_off = (r.pos + alignment - 1) // alignment * alignment
    return {"version": version, "metadata": meta, "tensors": tensors,
            "tensor_data_offset": data_off, "alignment": alignment}


def tensor_nbytes(t: dict) -> int:
    """GGUFTensorInfo::data_size (src/gguf_loader.rs:160-166)."""
    n = 1
    for d in t["dims"]:
        n *= d
    bs, epb = GGML_TYPES[t["type"]]
    return (n + epb - 1) // epb * bs


def build_gguf_bytes(metadata, tensors) -> bytes:
    """build_gguf_bytes (src/gguf_loader.rs:766-824): metadata is a list of
    (key, value_type, raw_value_bytes); tensors a list of (name, dims, type, data)."""
    buf = bytearray()
    buf += struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(metadata))
    for key, vt, raw in metadata:
        kb = key.encode()
        buf += struct.pack("<Q", len(kb)) + kb + struct.pack("<I", vt) + bytes(raw)
    off = 0
    blobs = []
    for name, dims, qt, data in tensors:
        nb = name.encode()
        buf += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims))
        for d in dims:
            buf += struct.pack("<Q", d)
        buf += struct.pack("<IQ", qt, off)
        off += len(data)
        blobs.append(bytes(data))
    pad = (GGUF_DEFAULT_ALIGNMENT - len(buf) % GGUF_DEFAULT_ALIGNMENT) % GGUF_DEFAULT_ALIGNMENT
    buf += bytes(pad)
    for b in blobs:
        buf += b
    return bytes(buf)
