"""GGUF reader and writer over libvxb.so.

Reader: host-side mirror of parse_gguf / get_tensor (src/gguf_loader.rs:341-408,
536-584) for the quantized path. The file is memory-mapped by the library;
Q4_0 / Q8_0 tensors upload as blocks into the tiled device layout (no f32
dequantization).

Writer (write_gguf): GGUF v3 files in the container format parse_gguf reads
(header, typed metadata, tensor descriptors, data from an aligned offset), for
synthetic models and exported weights. Q4_0 / Q8_0 tensors are packed by the
library's host block quantizer (vxb_pack_blocks_f32: the same codes as the
device quantizer and quantize_int4/int8 PerGroup 32); each tensor starts on an
alignment boundary of the data section.
"""
from __future__ import annotations

import ctypes
import os
import struct

import numpy as np

from . import _native as N

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q8_0 = 0, 1, 2, 3, 8

# GGUFValueType (src/gguf_loader.rs:21-36)
(GGUF_U8, GGUF_I8, GGUF_U16, GGUF_I16, GGUF_U32, GGUF_I32, GGUF_F32, GGUF_BOOL, GGUF_STRING, GGUF_ARRAY,
 GGUF_U64, GGUF_I64, GGUF_F64) = range(13)
GGUF_MAGIC = 0x46475547
GGUF_DEFAULT_ALIGNMENT = 32
# GGMLQuantType block geometry (src/gguf_loader.rs:61-128): type -> (bytes per block, elements per block)
GGML_BLOCKS = {0: (4, 1), 1: (2, 1), 2: (18, 32), 3: (20, 32), 6: (22, 32), 7: (24, 32), 8: (34, 32),
               10: (84, 256), 11: (110, 256), 12: (144, 256), 13: (176, 256), 14: (210, 256)}
_SCALAR_FMT = {GGUF_U8: "<B", GGUF_I8: "<b", GGUF_U16: "<H", GGUF_I16: "<h", GGUF_U32: "<I", GGUF_I32: "<i",
               GGUF_F32: "<f", GGUF_U64: "<Q", GGUF_I64: "<q", GGUF_F64: "<d"}


class GGUFError(N.VxbError):
    pass


def _check(rc):
    if rc != N.VXB_OK:
        raise GGUFError(rc, N.last_error(None))


class GGUFFile:
    """Open from a path (str) or parse bytes in memory (kept alive here)."""

    def __init__(self, source):
        L = N.lib()
        p = ctypes.c_void_p()
        if isinstance(source, (bytes, bytearray, memoryview)):
            self._buf = ctypes.create_string_buffer(bytes(source), len(source))
            _check(L.vxb_gguf_open_memory(self._buf, len(source), ctypes.byref(p)))
        else:
            self._buf = None
            _check(L.vxb_gguf_open(str(source).encode(), ctypes.byref(p)))
        self.ptr = p
        v, nt, nm, off, al = (ctypes.c_uint32(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_uint64(),
                              ctypes.c_uint64())
        _check(L.vxb_gguf_info(self.ptr, ctypes.byref(v), ctypes.byref(nt), ctypes.byref(nm), ctypes.byref(off),
                               ctypes.byref(al)))
        self.version, self.n_tensors, self.n_metadata = v.value, nt.value, nm.value
        self.tensor_data_offset, self.alignment = off.value, al.value

    def close(self):
        if getattr(self, "ptr", None):
            N.lib().vxb_gguf_close(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tensor_info(self, index: int) -> dict:
        name = ctypes.create_string_buffer(512)
        t, nd = ctypes.c_int(), ctypes.c_int()
        dims = (ctypes.c_uint64 * 4)()
        off, nb = ctypes.c_uint64(), ctypes.c_uint64()
        _check(N.lib().vxb_gguf_tensor(self.ptr, index, name, 512, ctypes.byref(t), ctypes.byref(nd), dims,
                                       ctypes.byref(off), ctypes.byref(nb), None))
        return {"name": name.value.decode(), "type": t.value, "dims": list(dims[:nd.value]), "offset": off.value,
                "nbytes": nb.value}

    def tensors(self) -> list[dict]:
        return [self.tensor_info(i) for i in range(self.n_tensors)]

    def find(self, name: str) -> int:
        i = ctypes.c_int64()
        _check(N.lib().vxb_gguf_find_tensor(self.ptr, name.encode(), ctypes.byref(i)))
        return i.value

    def tensor_bytes(self, name: str) -> np.ndarray:
        """A copy of the tensor's stored bytes (bounds-checked as get_tensor)."""
        i = self.find(name)
        nb = ctypes.c_uint64()
        ptr = ctypes.c_void_p()
        _check(N.lib().vxb_gguf_tensor(self.ptr, i, None, 0, None, None, None, None, ctypes.byref(nb),
                                       ctypes.byref(ptr)))
        return np.ctypeslib.as_array((ctypes.c_uint8 * nb.value).from_address(ptr.value)).copy()

    def meta_int(self, key: str) -> int:
        v = ctypes.c_int64()
        _check(N.lib().vxb_gguf_meta_int(self.ptr, key.encode(), ctypes.byref(v)))
        return v.value

    def meta_float(self, key: str) -> float:
        v = ctypes.c_double()
        _check(N.lib().vxb_gguf_meta_float(self.ptr, key.encode(), ctypes.byref(v)))
        return v.value

    def meta_string(self, key: str) -> str:
        n = ctypes.c_size_t()
        _check(N.lib().vxb_gguf_meta_string(self.ptr, key.encode(), None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(n.value + 1)
        _check(N.lib().vxb_gguf_meta_string(self.ptr, key.encode(), buf, n.value + 1, None))
        return buf.raw[:n.value].decode()

    def upload_tiled(self, name: str, device=None):
        """Q4_0 / Q8_0 tensor -> quant.TiledWeight on the GPU (rows = product of
        the dimensions after the first, K = the first)."""
        import torch

        from . import quant as Q
        i = self.find(name)
        info = self.tensor_info(i)
        if info["type"] not in (GGML_Q4_0, GGML_Q8_0):
            raise GGUFError(N.VXB_EUNSUPPORTED, f"tensor '{name}' is not Q4_0 / Q8_0")
        K = info["dims"][0]
        rows = int(np.prod(info["dims"][1:])) if len(info["dims"]) > 1 else 1
        ctx = Q.context(device)
        nbytes = N.lib().vxb_tiled_bytes(info["type"], rows, K)
        tiled = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{ctx.device}")
        ctx.call("vxb_gguf_upload_tiled", self.ptr, i, ctypes.c_void_p(tiled.data_ptr()), nbytes, Q._stream_ptr())
        return Q.TiledWeight.from_tiled(tiled, info["type"], rows, K)

    def upload(self, name: str, device=None):
        """Any tensor (F32, F16, Q4_0, Q4_1, Q8_0) as its GGUF bytes on the
        GPU, wrapped as a BlockRows (rows = product of the dimensions after the
        first, K = the first): dequantize() or gemv() over it on the device."""
        import torch

        from . import quant as Q
        i = self.find(name)
        info = self.tensor_info(i)
        K = info["dims"][0]
        rows = int(np.prod(info["dims"][1:])) if len(info["dims"]) > 1 else 1
        nbytes = N.lib().vxb_block_bytes(info["type"], rows * K)
        if nbytes == 0:
            raise GGUFError(N.VXB_EUNSUPPORTED, f"tensor '{name}' has ggml type {info['type']}")
        ctx = Q.context(device)
        buf = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{ctx.device}")
        ctx.call("vxb_gguf_upload", self.ptr, i, ctypes.c_void_p(buf.data_ptr()), nbytes, Q._stream_ptr())
        return Q.BlockRows(buf, info["type"], rows, K)



# ---------------------------------------------------------------- writer

class GGUFValue:
    """An explicitly typed metadata value (type: GGUF_U8 .. GGUF_F64). For
    GGUF_ARRAY the value is a list (element type inferred from its first item)
    or (element_type, items)."""

    __slots__ = ("type", "value")

    def __init__(self, type: int, value):
        if not 0 <= type <= 12:
            raise ValueError(f"unknown GGUF value type {type}")
        self.type, self.value = type, value


def _infer_type(v) -> int:
    if isinstance(v, (bool, np.bool_)):
        return GGUF_BOOL
    if isinstance(v, (int, np.integer)):
        return GGUF_U32 if 0 <= v < 2**32 else GGUF_I64
    if isinstance(v, (float, np.floating)):
        return GGUF_F32
    if isinstance(v, str):
        return GGUF_STRING
    if isinstance(v, (list, tuple)):
        return GGUF_ARRAY
    raise TypeError(f"no GGUF value type for {type(v).__name__}")


def _string(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t: int, v, elem_type=None) -> bytes:
    if t in _SCALAR_FMT:
        return struct.pack(_SCALAR_FMT[t], v)
    if t == GGUF_BOOL:
        return struct.pack("<B", 1 if v else 0)
    if t == GGUF_STRING:
        return _string(v)
    if t == GGUF_ARRAY:
        et = elem_type if elem_type is not None else (_infer_type(v[0]) if len(v) else GGUF_U32)
        if et == GGUF_ARRAY:
            raise TypeError("nested GGUF arrays are not written")
        return struct.pack("<IQ", et, len(v)) + b"".join(_value(et, x) for x in v)
    raise ValueError(f"unknown GGUF value type {t}")


def _typed(v):
    """(type, value, element type or None) of a metadata value."""
    if isinstance(v, GGUFValue):
        if v.type == GGUF_ARRAY and isinstance(v.value, tuple) and len(v.value) == 2 and \
                type(v.value[0]) is int and isinstance(v.value[1], (list, tuple)):
            return GGUF_ARRAY, v.value[1], v.value[0]
        return v.type, v.value, None
    return _infer_type(v), v, None


def _tensor_blob(name: str, data, ggml_type: int):
    """(dims, bytes) of one tensor. data: an array whose last axis is the row
    (GGUF dims are the shape reversed), or (dims, raw bytes)."""
    if isinstance(data, tuple) and len(data) == 2 and isinstance(data[1], (bytes, bytearray, memoryview)):
        dims, raw = [int(d) for d in data[0]], bytes(data[1])
        if ggml_type not in GGML_BLOCKS:
            raise ValueError(f"tensor '{name}': unknown ggml type {ggml_type}")
        bs, epb = GGML_BLOCKS[ggml_type]
        n = int(np.prod(dims)) if dims else 1
        if len(raw) != (n + epb - 1) // epb * bs:
            raise ValueError(f"tensor '{name}': {len(raw)} bytes for {n} elements of ggml type {ggml_type}")
        return dims, raw
    a = np.ascontiguousarray(np.asarray(data, dtype=np.float32))
    dims = [int(d) for d in reversed(a.shape)] or [1]
    if ggml_type == GGML_F32:
        return dims, a.tobytes()
    if ggml_type == GGML_F16:
        return dims, a.astype(np.float16).tobytes()
    if ggml_type in (GGML_Q4_0, GGML_Q8_0):
        if dims[0] % 32:
            raise ValueError(f"tensor '{name}': row length {dims[0]} is not a multiple of the 32-element block")
        n = a.size
        out = np.empty(n // 32 * (18 if ggml_type == GGML_Q4_0 else 34), dtype=np.uint8)
        _check(N.lib().vxb_pack_blocks_f32(ggml_type, a.ctypes.data_as(ctypes.c_void_p), n,
                                           out.ctypes.data_as(ctypes.c_void_p)))
        return dims, out.tobytes()
    raise ValueError(f"tensor '{name}': ggml type {ggml_type} is not written (F32, F16, Q4_0, Q8_0)")


def write_gguf(path, metadata=None, tensors=(), alignment: int = GGUF_DEFAULT_ALIGNMENT) -> bytes:
    """Build a GGUF v3 file and return its bytes; also write it to `path`
    (through a temporary file and a rename) unless path is None.

    metadata: dict or list of (key, value) pairs; a value is a bool, an int
    (U32 when it fits, else I64), a float (F32), a str, a list (ARRAY, element
    type from the first item) or a GGUFValue for an explicit type.
    tensors: (name, data, ggml_type) triples; data is a float array whose last
    axis is the row (GGUF dims = the shape reversed; Q4_0 / Q8_0 rows are a
    multiple of 32), or (dims, raw bytes) stored as given.
    alignment: alignment of the data section and of every tensor in it; a
    value other than 32 is recorded as general.alignment (U32). A
    general.alignment entry in metadata takes precedence.
    """
    items = list(metadata.items()) if isinstance(metadata, dict) else list(metadata or [])
    for k, v in items:
        if k == "general.alignment":
            alignment = int(v.value if isinstance(v, GGUFValue) else v)
            break
    else:
        if alignment != GGUF_DEFAULT_ALIGNMENT:
            items.append(("general.alignment", GGUFValue(GGUF_U32, alignment)))
    if alignment <= 0 or alignment & (alignment - 1):
        raise ValueError("alignment must be a power of two")
    meta = bytearray()
    for key, v in items:
        t, val, et = _typed(v)
        meta += _string(key) + struct.pack("<I", t) + _value(t, val, et)
    descs = bytearray()
    blobs = []
    off = 0
    for name, data, ggml_type in tensors:
        dims, raw = _tensor_blob(name, data, ggml_type)
        off = (off + alignment - 1) // alignment * alignment
        descs += _string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        descs += struct.pack("<IQ", ggml_type, off)
        blobs.append((off, raw))
        off += len(raw)
    head = struct.pack("<IIQQ", GGUF_MAGIC, 3, len(blobs), len(items)) + bytes(meta) + bytes(descs)
    data_off = (len(head) + alignment - 1) // alignment * alignment
    out = bytearray(head)
    for o, raw in blobs:
        out += bytes(data_off + o - len(out))
        out += raw
    if not blobs:
        out += bytes(data_off - len(out))
    out = bytes(out)
    if path is not None:
        tmp = f"{path}.tmp{os.getpid()}"
        with open(tmp, "wb") as fh:
            fh.write(out)
        os.replace(tmp, path)
    return out
