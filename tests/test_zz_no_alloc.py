"""vxb_gemv_q_static: the GEMV entry point that allocates no device memory.

It exists for callers that cannot call cudaMalloc (an embedding runtime that
owns all device memory, or code that must not grow its footprint mid-run): its
split-K scratch and error word live in a fixed array inside libvxb instead of
the context workspace. These tests call it through the C ABI twice in a row
per shape and check each result against the CPU oracle's dequantize-then-
matvec (f32 output, max relative error floored at 1e-3 of max|y| <= 1e-3) and
against vxb_gemv_q; the shapes cover the per-warp stream kernel, the group
kernel without a split, with a cluster reduction and with global partials in
the fixed array (the planner's choice is read back with vxb_gemv_plan_info).
A size beyond the array's limit is rejected, and a timeout recorded in the
array's error word is reported (and cleared) by vxb_device_error.

The file is collected last so that a run stopping at its first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests.parity import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

OFMT = {2: O.GGML_Q4_0, 8: O.GGML_Q8_0}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _plan(L, ctx, fmt, N, K, B, static):
    kern, splits, cl = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    rc = L.vxb_gemv_plan_info(ctx, fmt, N, K, B, int(static), ctypes.byref(kern), ctypes.byref(splits),
                              ctypes.byref(cl))
    assert rc == 0
    return kern.value, splits.value, cl.value


# (format, N, K, batch, expected path or None where the occupancy-driven
# planner may pick either): "stream" = per-warp stream kernel,
# "single" = group kernel without a split, "cluster" = group kernel whose
# splits add through distributed shared memory, "global" = group kernel whose
# splits add through partial sums in the fixed array, "tcgen05" = the
# tensor-core kernel (its splits add through distributed shared memory)
CASES = [("Q4_0", 4096, 4096, 1, "stream"), ("Q4_0", 11008, 4096, 3, "stream"),
         ("Q8_0", 1000, 160, 3, None), ("Q8_0", 11008, 4096, 4, None),
         ("Q4_0", 4096, 11008, 20, None), ("Q4_0", 1024, 16384, 16, "global"),
         ("Q4_0", 512, 8192, 12, "global"), ("Q8_0", 2048, 128, 5, "single"),
         ("Q8_0", 512, 8192, 9, "tcgen05"), ("Q4_0", 4096, 4096, 32, "tcgen05")]


def _path(kern, splits, cl):
    if kern == 0:
        return "stream"
    if kern == 2:
        return "tcgen05"
    return "single" if splits == 1 else ("cluster" if cl else "global")


@pytest.mark.parametrize("fmt_name,N,K,B,path", CASES)
def test_static_scratch_gemv_matches_oracle(cuda_ok, fmt_name, N, K, B, path):
    from vortex_b200 import _native as NAT
    from vortex_b200 import quant as Q
    fmt = getattr(NAT, fmt_name)
    rng = np.random.default_rng(N + K + B)
    w = rng.normal(0.0, 0.02, (N, K)).astype(np.float32)
    xbits = O.f32_array_to_bf16_bits(rng.standard_normal((B, K)).astype(np.float32))
    xf = O.bf16_bits_to_f32_array(xbits).reshape(B, K).astype(np.float64)
    ref = O.gemv_blocks(OFMT[fmt], O.quantize_blocks(OFMT[fmt], w.astype(np.float64)), N, K, xf)
    tw = Q.TiledWeight.from_float(torch.from_numpy(w).cuda(), fmt)
    x = torch.from_numpy(xbits.view(np.int16)).cuda().view(torch.bfloat16).reshape(B, K)
    L = NAT.lib()
    got_path = _path(*_plan(L, tw.ctx.ptr, fmt, N, K, B, True))
    if path is not None:
        assert got_path == path, (got_path, path)
    alloc = tw.gemv(x).cpu().numpy()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        y = torch.full((B, N), float("nan"), device="cuda")
        rc = L.vxb_gemv_q_static(tw.ctx.ptr, fmt, _ptr(tw.tiled), N, K, _ptr(x), B, NAT.F32, _ptr(y), stream)
        assert rc == NAT.VXB_OK, NAT.last_error(tw.ctx.ptr)
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert rel_err(got, ref) <= 1e-3, (call, got_path, rel_err(got, ref))
        assert rel_err(got, alloc) <= 1e-3, (call, got_path)
    err = ctypes.c_int(-1)
    assert L.vxb_device_error(tw.ctx.ptr, ctypes.byref(err)) == NAT.VXB_OK and err.value == 0


def test_static_scratch_gemv_rejects_sizes_beyond_the_limit(cuda_ok):
    from vortex_b200 import _native as NAT
    from vortex_b200 import quant as Q
    N, K, B = 40000, 64, 32  # 32 * 40000 > 1048576
    tw = Q.TiledWeight.from_float(torch.zeros(N, K, device="cuda"), "Q4_0")
    x = torch.zeros(B, K, device="cuda", dtype=torch.bfloat16)
    y = torch.zeros(B, N, device="cuda")
    L = NAT.lib()
    rc = L.vxb_gemv_q_static(tw.ctx.ptr, NAT.Q4_0, _ptr(tw.tiled), N, K, _ptr(x), B, NAT.F32, _ptr(y), None)
    assert rc == NAT.VXB_EINVAL
    assert "static scratch limit" in NAT.last_error(tw.ctx.ptr)


def test_static_error_word_is_reported_and_cleared(cuda_ok):
    """A wait that runs out while writing the fixed array's error word (the
    library's mbarrier wait on a barrier nobody arrives on, 2^20 cycles) is
    reported by vxb_device_error as VXB_ETIMEOUT, the word is cleared, and the
    static GEMV still computes the right product afterwards."""
    from vortex_b200 import _native as NAT
    from vortex_b200 import quant as Q
    N, K, B = 1024, 256, 4
    rng = np.random.default_rng(5)
    w = rng.normal(0.0, 0.02, (N, K)).astype(np.float32)
    tw = Q.TiledWeight.from_float(torch.from_numpy(w).cuda(), "Q8_0")
    ctx = tw.ctx.ptr
    L = NAT.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.vxb_selftest_wait_timeout(ctx, 0, 1, 1 << 20, stream) == NAT.VXB_OK, NAT.last_error(ctx)
    err = ctypes.c_int(0)
    assert L.vxb_device_error(ctx, ctypes.byref(err)) == NAT.VXB_ETIMEOUT
    assert err.value != 0
    assert L.vxb_device_error(ctx, ctypes.byref(err)) == NAT.VXB_OK and err.value == 0
    x = torch.randn(B, K, device="cuda").bfloat16()
    y = torch.zeros(B, N, device="cuda")
    rc = L.vxb_gemv_q_static(ctx, NAT.Q8_0, _ptr(tw.tiled), N, K, _ptr(x), B, NAT.F32, _ptr(y), stream)
    assert rc == NAT.VXB_OK
    assert rel_err(y.cpu().numpy(), tw.gemv(x).cpu().numpy()) <= 1e-3
