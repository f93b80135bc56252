"""CPU-only checks of the C ABI: the library loads, exports every entry point
declared in include/vxb.h, and its host-side block codec is bit-exact with the
oracle. No compute call needs a GPU here."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from vortex_b200 import _native as N
from vortex_b200 import quant as Q


def test_library_loads_and_exports_header_symbols():
    L = N.lib()
    names = N.header_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, f"declared in vxb.h but not exported: {missing}"
    # every declared symbol has a ctypes signature in the binding
    assert set(names) <= set(N.SIGNATURES), set(names) - set(N.SIGNATURES)
    assert L.vxb_abi_version() == 1


@pytest.mark.parametrize("fmt,ofmt", [(Q.Q4_0, O.GGML_Q4_0), (Q.Q8_0, O.GGML_Q8_0)])
@pytest.mark.parametrize("n", [32, 96, 1000, 4096 * 3])
def test_host_pack_bit_exact_vs_oracle(fmt, ofmt, n):
    rng = np.random.default_rng(n)
    w = rng.normal(0, 0.02, n).astype(np.float32)
    w[:7] = 0.0  # an all-zero-prefix group stays well defined
    got = Q.pack_blocks(fmt, w)
    want = O.quantize_blocks(ofmt, w.astype(np.float64))
    assert got.dtype == np.uint8 and np.array_equal(got, want)
    deq = Q.unpack_blocks(fmt, got, n)
    assert np.array_equal(deq, O.dequantize_blocks(ofmt, want, n))


@pytest.mark.parametrize("fmt,ofmt", [(Q.Q4_0, O.GGML_Q4_0), (Q.Q8_0, O.GGML_Q8_0)])
def test_host_pack_edge_values(fmt, ofmt):
    # zero groups (scale 1.0), exact ties (round half away from zero), huge and
    # tiny magnitudes (f16 truncation overflow / subnormal scales), NaN
    w = np.zeros(32 * 6, dtype=np.float64)
    w[32:64] = np.linspace(-1.0, 1.0, 32)
    w[64:96] = 1e6 * np.sign(np.arange(32) - 15.5)
    w[96:128] = 1e-7 * (np.arange(32) - 16)
    w[128:160] = [0.5, -0.5, 1.5, -1.5] * 8
    w[160] = np.nan
    w[161:192] = 0.25
    got = Q.pack_blocks(fmt, w)
    want = O.quantize_blocks(ofmt, w)
    assert np.array_equal(got, want)
    assert np.array_equal(Q.unpack_blocks(fmt, got, w.size), O.dequantize_blocks(ofmt, want, w.size),
                          equal_nan=True)


def test_error_codes_without_gpu():
    L = N.lib()
    out = np.zeros(64, dtype=np.uint8)
    w = np.zeros(32, dtype=np.float32)
    rc = L.vxb_pack_blocks_f32(99, w.ctypes.data_as(ctypes.c_void_p), 32, out.ctypes.data_as(ctypes.c_void_p))
    assert rc == N.VXB_EINVAL
    assert "unknown block format" in N.last_error(None)
    assert L.vxb_tiled_bytes(Q.Q4_0, 16, 33) == 0  # K must be a multiple of 32
    assert L.vxb_block_bytes(Q.Q4_0, 33) == 36 and L.vxb_block_bytes(Q.Q8_0, 64) == 68
    rc = L.vxb_init(0, None)
    assert rc == N.VXB_EINVAL
    with pytest.raises(N.VxbError):
        Q.pack_blocks("INT3", w)
