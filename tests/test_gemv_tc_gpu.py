"""K1 batches 9-32 through the tcgen05 kernel vs the CPU oracle. The routing
switch VXB_GEMV_TCGEN05 is read once per process, so the forced checks run in
a child process with it set; the default routing (which shapes take the
kernel) is read back with vxb_gemv_plan_info. Tolerance as for the other GEMV paths: max
relative error (floored at 1e-3 of max|y|) <= 1e-3 for f32 output.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import numpy as np, torch
from oracle import oracle as O
from tests.parity import rel_err
from vortex_b200 import quant as Q
OFMT = {2: O.GGML_Q4_0, 8: O.GGML_Q8_0}
fails = []
for fmt in (2, 8):
    for (N, K) in ((1000, 160), (300, 4096), (11008, 4096), (4096, 11008), (12288, 4096), (22016, 4096)):
        for B in (9, 17, 32):
            rng = np.random.default_rng(N + K + B)
            w = rng.normal(0.0, 0.02, (N, K)).astype(np.float32)
            x = rng.standard_normal((B, K)).astype(np.float32)
            xbits = O.f32_array_to_bf16_bits(x)
            xf = O.bf16_bits_to_f32_array(xbits).reshape(B, K)
            tw = Q.TiledWeight.from_float(torch.from_numpy(w).cuda(), fmt)
            xd = torch.from_numpy(xbits.view(np.int16)).cuda().view(torch.bfloat16).reshape(B, K)
            y = tw.gemv(xd).float().cpu().numpy()
            blocks = O.quantize_blocks(OFMT[fmt], w.astype(np.float64))
            ref = O.gemv_blocks(OFMT[fmt], blocks, N, K, xf.astype(np.float64))
            for b in range(B):
                e = rel_err(y[b], ref[b])
                if not e <= 1e-3:
                    fails.append((fmt, N, K, B, b, float(e)))
print("FAILS", fails)
assert not fails
'''


def test_gemv_tcgen05_matches_oracle(cuda_ok):
    env = dict(os.environ, VXB_GEMV_TCGEN05="1")
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]


@pytest.mark.parametrize("fmt_name,N,K,B,kernel", [
    ("Q4_0", 4096, 4096, 32, 2), ("Q4_0", 11008, 4096, 16, 1), ("Q4_0", 12288, 4096, 32, 2),
    ("Q4_0", 22016, 4096, 32, 2), ("Q4_0", 32000, 4096, 32, 2), ("Q4_0", 32000, 4096, 24, 1),
    ("Q8_0", 4096, 4096, 9, 2), ("Q8_0", 32000, 4096, 9, 2), ("Q8_0", 22016, 4096, 16, 1)])
def test_gemv_default_routing(cuda_ok, fmt_name, N, K, B, kernel):
    """Default routing by measurement: 2 = tcgen05 kernel, 1 = group kernel."""
    import ctypes
    if os.environ.get("VXB_GEMV_TCGEN05"):
        pytest.skip("routing forced by VXB_GEMV_TCGEN05")
    from vortex_b200 import _native as NAT
    from vortex_b200 import quant as Q
    import torch
    tw = Q.TiledWeight.from_float(torch.zeros(16, 32, device="cuda"), fmt_name)
    k, s_, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    assert NAT.lib().vxb_gemv_plan_info(tw.ctx.ptr, getattr(NAT, fmt_name), N, K, B, 0, ctypes.byref(k),
                                        ctypes.byref(s_), ctypes.byref(c)) == 0
    assert k.value == kernel, (k.value, s_.value)
