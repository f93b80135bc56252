"""GGUF reader over libvxb.so: host-side mirror of parse_gguf / get_tensor
(src/gguf_loader.rs:341-408, 536-584) for the quantized path. The file is
memory-mapped by the library; Q4_0 / Q8_0 tensors upload as blocks into the
tiled device layout (no f32 dequantization)."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native as N

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q8_0 = 0, 1, 2, 3, 8


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
