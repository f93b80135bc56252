"""GGUF Q4_0 / Q8_0 tensors uploaded into the tiled device layout without an
f32 dequantization: the untiled blocks equal the file's bytes, and the GEMV
over the uploaded weights matches the oracle's (src/gguf_loader.rs:413-498
dequantization, f64 matvec) with the GEMV gate (1e-3, f32 output)."""
import numpy as np
import pytest

from oracle import gguf_oracle as G
from oracle import oracle as O
from tests.parity import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("qt,ofmt", [(2, O.GGML_Q4_0), (8, O.GGML_Q8_0)])
def test_gguf_upload_tiled_and_gemv(cuda_ok, qt, ofmt):
    from vortex_b200 import gguf
    N, K = 300, 256
    rng = np.random.default_rng(qt)
    blocks = O.quantize_blocks(ofmt, rng.normal(0, 0.02, N * K))
    data = G.build_gguf_bytes([], [("w", [K, N], qt, bytes(blocks))])
    f = gguf.GGUFFile(data)
    tw = f.upload_tiled("w")
    assert np.array_equal(tw.to_blocks().cpu().numpy(), np.frombuffer(bytes(blocks), np.uint8))
    xb = O.f32_array_to_bf16_bits(rng.standard_normal((4, K)).astype(np.float32))
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16).reshape(4, K)
    y = tw.gemv(x).cpu().numpy()
    ref = O.gemv_blocks(ofmt, blocks, N, K, O.bf16_bits_to_f32_array(xb).reshape(4, K).astype(np.float64))
    assert rel_err(y, ref) <= 1e-3
