"""ctypes binding of libvxb.so (the C ABI declared in include/vxb.h).

The library is the product: there is no CPU fallback. If libvxb.so is missing
or fails to load, every entry point raises VxbError.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libvxb.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "vxb.h")

VXB_OK = 0
VXB_EINVAL = -1
VXB_ECUDA = -2
VXB_ENOMEM = -3
VXB_ETIMEOUT = -4
VXB_EFORMAT = -5
VXB_ENOBLOCKS = -6
VXB_EUNSUPPORTED = -7
VXB_ENCCL = -8

Q4_0 = 2
Q8_0 = 8
Q4_1 = 3
GGML_F32, GGML_F16 = 0, 1
F32, BF16, F16, I8 = 0, 1, 2, 3

_STATUS_NAMES = {0: "VXB_OK", -1: "VXB_EINVAL", -2: "VXB_ECUDA", -3: "VXB_ENOMEM", -4: "VXB_ETIMEOUT",
                 -5: "VXB_EFORMAT", -6: "VXB_ENOBLOCKS", -7: "VXB_EUNSUPPORTED", -8: "VXB_ENCCL"}


class VxbError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{_STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_I64 = ctypes.c_int64

# name -> (restype, argtypes); kept in the order of include/vxb.h
SIGNATURES = {
    "vxb_abi_version": (_I, []),
    "vxb_device_count": (_I, [ctypes.POINTER(_I)]),
    "vxb_init": (_I, [_I, ctypes.POINTER(_P)]),
    "vxb_destroy": (_I, [_P]),
    "vxb_last_error": (ctypes.c_char_p, [_P]),
    "vxb_alloc": (_I, [_P, _SZ, ctypes.POINTER(_P)]),
    "vxb_free": (_I, [_P, _P]),
    "vxb_memcpy_h2d": (_I, [_P, _P, _P, _SZ, _P]),
    "vxb_memcpy_d2h": (_I, [_P, _P, _P, _SZ, _P]),
    "vxb_memset": (_I, [_P, _P, _I, _SZ, _P]),
    "vxb_sync": (_I, [_P, _P]),
    "vxb_device_error": (_I, [_P, ctypes.POINTER(_I)]),
    "vxb_selftest_wait_timeout": (_I, [_P, _I, _I, ctypes.c_longlong, _P]),
    "vxb_block_bytes": (_SZ, [_I, _SZ]),
    "vxb_pack_blocks_f64": (_I, [_I, _P, _SZ, _P]),
    "vxb_pack_blocks_f32": (_I, [_I, _P, _SZ, _P]),
    "vxb_unpack_blocks": (_I, [_I, _P, _SZ, _P]),
    "vxb_quantize_blocks": (_I, [_P, _I, _P, _SZ, _P, _P]),
    "vxb_dequantize_blocks": (_I, [_P, _I, _P, _SZ, _P, _P]),
    "vxb_qt_data_bytes": (_SZ, [_I, _SZ]),
    "vxb_qt_num_groups": (_SZ, [_SZ, _SZ]),
    "vxb_qt_quantize": (_I, [_I, _P, _SZ, _SZ, _P, _P, _P]),
    "vxb_qt_mean_scale": (_I, [_P, _SZ, _P]),
    "vxb_quant_matmul": (_I, [_P, _I, _P, _P, _I, _I, _I, ctypes.c_double, ctypes.c_double, _I64, _I64, _P, _P]),
    "vxb_tiled_bytes": (_SZ, [_I, _I, _I]),
    "vxb_tile_weights": (_I, [_P, _I, _P, _I, _I, _P, _P]),
    "vxb_untile_weights": (_I, [_P, _I, _P, _I, _I, _P, _P]),
    "vxb_gemv_q": (_I, [_P, _I, _P, _I, _I, _P, _I, _I, _P, _P]),
    "vxb_gemv_blocks": (_I, [_P, _I, _P, _I, _I, _P, _I, _I, _P, _P]),
    "vxb_gemv_q_static": (_I, [_P, _I, _P, _I, _I, _P, _I, _I, _P, _P]),
    "vxb_gemv_plan_info": (_I, [_P, _I, _I, _I, _I, _I, _P, _P, _P]),
    "vxb_kv_create": (_I, [_P, _I, _I, _I, _I, _I, _I, _I, _I, ctypes.POINTER(_P)]),
    "vxb_kv_destroy": (_I, [_P]),
    "vxb_kv_append": (_I, [_P, _I, _I, _P, _P, _P, _P]),
    "vxb_kv_append_seq": (_I, [_P, _I, _I64, _I, _P, _P, _P]),
    "vxb_kv_free_seq": (_I, [_P, _I64]),
    "vxb_kv_fork": (_I, [_P, _I64, _I64, _I64, _P]),
    "vxb_kv_stats": (_I, [_P, _P]),
    "vxb_kv_seq_len": (_I, [_P, _I, _I64, _P]),
    "vxb_kv_block_table": (_I, [_P, _I, _I64, _P, _I, _P]),
    "vxb_kv_gather": (_I, [_P, _I, _I64, _P, _P, _P]),
    "vxb_decode_attention": (_I, [_P, _I, _I, _P, _P, _I, ctypes.c_float, _P, _P, _P]),
    "vxb_gemm_q": (_I, [_P, _I, _P, _I, _I, _P, _I, _I, _P, _P]),
    "vxb_flash_fwd": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, ctypes.c_float, _I, _P, _P, _P]),
    "vxb_flash_bwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, ctypes.c_float, _I, _P, _P, _P, _P]),
    "vxb_rmsnorm": (_I, [_P, _P, _P, _P, _I, _I, ctypes.c_float, _P, _P]),
    "vxb_swiglu": (_I, [_P, _P, _I, _I, _P, _P]),
    "vxb_argmax": (_I, [_P, _P, _I, _I, _P, _P]),
    "vxb_rope": (_I, [_P, _P, _I, _I, _P, _I, _P, _P]),
    "vxb_rope_angles": (_I, [_P, _P, _I, _I, _P, _I, _P, _P]),
    "vxb_add": (_I, [_P, _P, _P, _SZ, _P, _P]),
    "vxb_sample_top_p": (_I, [_P, _P, _I, _I, ctypes.c_double, ctypes.c_double, _P, _P, _P]),
    "vxb_batcher_create": (_I, [_I, ctypes.POINTER(_P)]),
    "vxb_batcher_destroy": (_I, [_P]),
    "vxb_batcher_add": (_I, [_P, _P, _SZ, ctypes.POINTER(_I)]),
    "vxb_batcher_remove": (_I, [_P, _I]),
    "vxb_batcher_num_active": (_I, [_P, ctypes.POINTER(_I)]),
    "vxb_batcher_slot": (_I, [_P, _I, _P, _P, _P, _P, _P]),
    "vxb_batcher_advance": (_I, [_P, _I, _I64, _I]),
    "vxb_nccl_unique_id": (_I, [_P]),
    "vxb_comm_init": (_I, [_P, _I, _I, _P, ctypes.POINTER(_P)]),
    "vxb_comm_destroy": (_I, [_P]),
    "vxb_allreduce_sum": (_I, [_P, _P, _SZ, _I, _P]),
    "vxb_decoder_create": (_I, [_P, _P, ctypes.POINTER(_P)]),
    "vxb_decoder_create_tp": (_I, [_P, _P, _P, ctypes.POINTER(_P)]),
    "vxb_decoder_destroy": (_I, [_P]),
    "vxb_decoder_init_random": (_I, [_P, ctypes.c_uint64, ctypes.c_float]),
    "vxb_decoder_set_weight": (_I, [_P, _I, _I, _P, _SZ]),
    "vxb_decoder_step": (_I, [_P, _I, _P, _P, _P, _P]),
    "vxb_decoder_prefill": (_I, [_P, _I64, _P, _I, _P, _P]),
    "vxb_decoder_step_device": (_I, [_P, _I, _P, _P, _P, _P]),
    "vxb_decoder_logits": (_I, [_P, _I, _P, _P]),
    "vxb_decoder_free_seq": (_I, [_P, _I64]),
    "vxb_decoder_fork": (_I, [_P, _I64, _I64, _I64]),
    "vxb_decoder_kv": (_I, [_P, ctypes.POINTER(_P)]),
    "vxb_decoder_stream": (_I, [_P, ctypes.POINTER(_P)]),
    "vxb_gguf_open": (_I, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    "vxb_gguf_open_memory": (_I, [_P, _SZ, ctypes.POINTER(_P)]),
    "vxb_gguf_close": (_I, [_P]),
    "vxb_gguf_info": (_I, [_P, _P, _P, _P, _P, _P]),
    "vxb_gguf_tensor": (_I, [_P, _I64, _P, _SZ, _P, _P, _P, _P, _P, _P]),
    "vxb_gguf_find_tensor": (_I, [_P, ctypes.c_char_p, _P]),
    "vxb_gguf_meta_int": (_I, [_P, ctypes.c_char_p, _P]),
    "vxb_gguf_meta_float": (_I, [_P, ctypes.c_char_p, _P]),
    "vxb_gguf_meta_string": (_I, [_P, ctypes.c_char_p, _P, _SZ, _P]),
    "vxb_gguf_upload_tiled": (_I, [_P, _P, _I64, _P, _SZ, _P]),
    "vxb_gguf_upload": (_I, [_P, _P, _I64, _P, _SZ, _P]),
    "vxb_tmodel_create": (_I, [_P, _P, ctypes.POINTER(_P)]),
    "vxb_tmodel_destroy": (_I, [_P]),
    "vxb_tmodel_param_count": (_I, [_P, ctypes.POINTER(_SZ)]),
    "vxb_tmodel_set_params": (_I, [_P, _P, _SZ]),
    "vxb_tmodel_get_params": (_I, [_P, _P, _SZ]),
    "vxb_tmodel_forward": (_I, [_P, _P, _I, _P, _P]),
}

_lib = None
_load_error = None


def header_symbols() -> list[str]:
    """Names of every entry point declared in include/vxb.h."""
    with open(HEADER) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"\b(vxb_[a-z0-9_]+)\s*\(", text)


def lib():
    """Load libvxb.so (raises VxbError if it is missing: there is no fallback)."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise VxbError(VXB_EUNSUPPORTED, f"{LIB_PATH} is missing; build it with `python -m vortex_b200.build`")
    try:
        L = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
    except OSError as e:
        raise VxbError(VXB_EUNSUPPORTED, f"cannot load {LIB_PATH}: {e}")
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error(ctx=None) -> str:
    s = lib().vxb_last_error(ctx)
    return s.decode() if s else ""


def check(rc: int, ctx=None) -> int:
    if rc != VXB_OK:
        raise VxbError(rc, last_error(ctx))
    return rc


class Context:
    """One vxb_ctx per device (vxb_init / vxb_destroy)."""

    _by_device: dict[int, "Context"] = {}

    def __init__(self, device: int = 0):
        L = lib()
        p = ctypes.c_void_p()
        check(L.vxb_init(device, ctypes.byref(p)))
        self.ptr = p
        self.device = device

    @classmethod
    def get(cls, device: int = 0) -> "Context":
        c = cls._by_device.get(device)
        if c is None:
            c = cls(device)
            cls._by_device[device] = c
        return c

    def call(self, name: str, *args) -> int:
        rc = getattr(lib(), name)(self.ptr, *args)
        if rc != VXB_OK:
            raise VxbError(rc, last_error(self.ptr))
        return rc

    def close(self):
        if self.ptr:
            lib().vxb_destroy(self.ptr)
            self.ptr = None
            Context._by_device.pop(self.device, None)
