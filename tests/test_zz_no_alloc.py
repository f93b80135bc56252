"""vxb_gemv_q_static: the GEMV entry point that allocates no device memory.

It exists for callers that cannot call cudaMalloc (an embedding runtime that
owns all device memory, or code that must not grow its footprint mid-run): its
split-K scratch lives in a fixed array inside libvxb instead of the context
workspace. This test calls it through the C ABI twice in a row and checks each
result against vxb_gemv_q (f32 output, max relative error floored at 1e-3 of
max|y| <= 1e-3), and that a size beyond the array's limit is rejected.
"""
import ctypes

import numpy as np
import pytest

from tests.parity import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("fmt_name,N,K,B", [("Q4_0", 4096, 4096, 1), ("Q8_0", 11008, 4096, 4),
                                            ("Q4_0", 4096, 11008, 32), ("Q8_0", 1000, 160, 3),
                                            ("Q4_0", 11008, 4096, 3)])
def test_static_scratch_gemv_matches_allocating_gemv(cuda_ok, fmt_name, N, K, B):
    from vortex_b200 import _native as NAT
    from vortex_b200 import quant as Q
    fmt = getattr(NAT, fmt_name)
    g = torch.Generator(device="cuda").manual_seed(N + K + B)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.02
    tw = Q.TiledWeight.from_float(w, fmt)
    x = torch.randn(B, K, device="cuda", generator=g).bfloat16()
    ref = tw.gemv(x).cpu().numpy()
    L = NAT.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        y = torch.full((B, N), float("nan"), device="cuda")
        rc = L.vxb_gemv_q_static(tw.ctx.ptr, fmt, _ptr(tw.tiled), N, K, _ptr(x), B, NAT.F32, _ptr(y), stream)
        assert rc == NAT.VXB_OK, NAT.last_error(tw.ctx.ptr)
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert rel_err(got, ref) <= 1e-3, (call, rel_err(got, ref))


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
