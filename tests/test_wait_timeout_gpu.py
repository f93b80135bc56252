"""Bounded device waits run out into an error status, not a hang.

Every wait in the library's kernels is bounded: the mbarrier phases of the
K1-K4 stage rings and the peer-slot polls of the one-shot all-reduce give up
after a cycle budget, set the context's device error word and let the kernel
finish (the heartbeat-timeout semantics of src/dist_runtime.rs:426-456: a
peer that never answers becomes an error, not a stall). vxb_selftest_wait_
timeout runs those same helpers on a barrier nobody arrives on and a slot
nobody fills, with a short budget; vxb_device_error must then return
VXB_ETIMEOUT once, the next call VXB_OK, and the context must stay usable.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("kind", [0, 1], ids=["mbarrier", "peer_slot"])
def test_wait_runs_out_and_is_reported(cuda_ok, kind):
    from vortex_b200 import _native as NAT
    from vortex_b200 import quant as Q
    ctx = Q.context().ptr
    L = NAT.lib()
    err = ctypes.c_int(0)
    L.vxb_device_error(ctx, ctypes.byref(err))  # start from a clear word
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.vxb_selftest_wait_timeout(ctx, kind, 0, 1 << 21, stream)
    assert rc == NAT.VXB_OK, NAT.last_error(ctx)
    assert L.vxb_device_error(ctx, ctypes.byref(err)) == NAT.VXB_ETIMEOUT
    assert err.value == 1
    assert "timed out" in NAT.last_error(ctx)
    assert L.vxb_device_error(ctx, ctypes.byref(err)) == NAT.VXB_OK and err.value == 0
    # the context still computes
    w = torch.randn(256, 128, device="cuda") * 0.02
    tw = Q.TiledWeight.from_float(w, "Q4_0")
    x = torch.randn(1, 128, device="cuda").bfloat16()
    y = tw.gemv(x)
    torch.cuda.synchronize()
    assert np.all(np.isfinite(y.cpu().numpy()))
    assert L.vxb_device_error(ctx, ctypes.byref(err)) == NAT.VXB_OK


def test_selftest_rejects_bad_arguments(cuda_ok):
    from vortex_b200 import _native as NAT
    from vortex_b200 import quant as Q
    ctx = Q.context().ptr
    L = NAT.lib()
    assert L.vxb_selftest_wait_timeout(ctx, 2, 0, 1000, None) == NAT.VXB_EINVAL
    assert L.vxb_selftest_wait_timeout(ctx, 0, 0, 0, None) == NAT.VXB_EINVAL
    assert L.vxb_selftest_wait_timeout(ctx, 0, 0, (1 << 31) + 1, None) == NAT.VXB_EINVAL
