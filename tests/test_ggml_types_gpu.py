"""GGUF tensor types beyond the tiled formats on the device (a8): device
dequantization bit-identical with the oracle for F32 / F16 / Q4_0 / Q4_1 /
Q8_0, and a GGUF file holding Q4_1 and F16 projections uploaded as its rows
(vxb_gguf_upload, no conversion) and multiplied by vxb_gemv_blocks: f32
output within 1e-3 (floored relative error) of the oracle's dequantize +
f64 matvec."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.parity import rel_err
from tests.test_ggml_types_cpu import q4_1_blocks

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("kind", ["Q4_1", "F16", "F32", "Q4_0", "Q8_0"])
def test_device_dequantize_bit_exact(cuda_ok, kind):
    from vortex_b200 import _native as N
    from vortex_b200 import quant as Q
    rng = np.random.default_rng(7)
    n = 4096 - 7 if kind in ("F16", "F32") else 4096
    if kind == "Q4_1":
        raw, t, ot = q4_1_blocks(rng, n // 32, subnormal=True), N.Q4_1, O.GGML_Q4_1
    elif kind == "F16":
        h = rng.integers(0, 0x7C00, size=n, dtype=np.uint16)
        raw, t, ot = h.view(np.uint8), N.GGML_F16, O.GGML_F16
    elif kind == "F32":
        raw, t, ot = rng.standard_normal(n).astype(np.float32).view(np.uint8), N.GGML_F32, O.GGML_F32
    else:
        ot = O.GGML_Q4_0 if kind == "Q4_0" else O.GGML_Q8_0
        raw, t = O.quantize_blocks(ot, rng.standard_normal(n) * 0.1), getattr(N, kind)
    d = torch.from_numpy(np.ascontiguousarray(raw)).cuda()
    rows = Q.BlockRows(d, t, 1, n)
    got = rows.dequantize().cpu().numpy().ravel()
    want = O.dequantize_blocks(ot, raw, n)
    assert np.array_equal(got.view(np.uint32), np.asarray(want, np.float32).view(np.uint32))


@pytest.mark.parametrize("B", [1, 5, 17])
def test_gguf_q4_1_and_f16_projections(cuda_ok, tmp_path, B):
    from vortex_b200 import gguf as G
    rng = np.random.default_rng(B)
    N_, K = 1000, 4096
    q41 = q4_1_blocks(rng, N_ * K // 32)
    f16 = (rng.standard_normal((N_, K)) * 0.02).astype(np.float16)
    path = str(tmp_path / "m.gguf")
    G.write_gguf(path, {"general.architecture": "llama"},
                 [("blk.0.ffn_up.weight", ([K, N_], q41.tobytes()), G.GGML_Q4_1),
                  ("blk.0.attn_q.weight", ([K, N_], f16.view(np.uint8).tobytes()), G.GGML_F16)])
    f = G.GGUFFile(path)
    x = torch.randn(B, K, device="cuda").bfloat16()
    xf = x.float().cpu().numpy().astype(np.float64)
    for name, raw, ot in (("blk.0.ffn_up.weight", q41, O.GGML_Q4_1),
                          ("blk.0.attn_q.weight", f16.view(np.uint8).ravel(), O.GGML_F16)):
        w = f.upload(name)
        assert (w.N, w.K) == (N_, K)
        y = w.gemv(x).cpu().numpy()
        deq = O.dequantize_blocks(ot, raw, N_ * K).astype(np.float64).reshape(N_, K)
        ref = xf @ deq.T
        assert rel_err(y, ref) <= 1e-3, (name, rel_err(y, ref))
    f.close()
