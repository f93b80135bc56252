"""K2 prefill GEMM (tcgen05, exact bf16 hi + lo weights) against the oracle's
restatement of weight_only_matmul (dequantize then f64 matmul,
src/quantize.rs:845-852, 890-902).

Gate: f32 output, max relative error floored at 1e-3 of max|y| <= 1e-3;
bf16 output <= 1e-2.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.parity import norm_err, rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

OFMT = {2: O.GGML_Q4_0, 8: O.GGML_Q8_0}


def _case(fmt, M, N, K, seed, out_dtype=None, rows=None):
    from vortex_b200 import quant as Q
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, (N, K)).astype(np.float32)
    xb = O.f32_array_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
    xf = O.bf16_bits_to_f32_array(xb).reshape(M, K)
    tw = Q.TiledWeight.from_float(torch.from_numpy(w).cuda(), fmt)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16).reshape(M, K)
    y = tw.gemm(x, out_dtype=out_dtype).float().cpu().numpy()
    rows = np.arange(M) if rows is None else rows
    blocks = O.quantize_blocks(OFMT[fmt], w.astype(np.float64))
    ref = O.gemv_blocks(OFMT[fmt], blocks, N, K, xf[rows].astype(np.float64))
    return y[rows], ref


@pytest.mark.parametrize("fmt", [2, 8])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (33, 17, 32), (300, 1000, 160), (257, 300, 4096)])
def test_gemm_matches_oracle(cuda_ok, fmt, M, N, K):
    y, ref = _case(fmt, M, N, K, seed=M + N + K)
    assert rel_err(y, ref) <= 1e-3, (rel_err(y, ref), norm_err(y, ref))


@pytest.mark.parametrize("fmt", [2, 8])
def test_gemm_prefill_shape_sampled_rows(cuda_ok, fmt):
    """2048 prompt rows x the 7B gate/up projection (11008 x 4096): 16 rows
    checked against the oracle."""
    rows = np.array([0, 1, 2, 127, 128, 255, 511, 777, 1024, 1500, 1800, 2000, 2045, 2046, 2047, 1023])
    y, ref = _case(fmt, 2048, 11008, 4096, seed=3, rows=rows)
    assert rel_err(y, ref) <= 1e-3, (rel_err(y, ref), norm_err(y, ref))


def test_gemm_bf16_output(cuda_ok):
    y, ref = _case(2, 200, 512, 256, seed=9, out_dtype=torch.bfloat16)
    assert rel_err(y, ref) <= 1e-2


def test_weight_only_matmul_routes_by_rows(cuda_ok):
    """weight_only_matmul: <= 32 rows through the GEMV, more through the GEMM;
    both agree with the oracle."""
    from vortex_b200 import quant as Q
    rng = np.random.default_rng(4)
    N, K = 384, 512
    w = rng.normal(0.0, 0.02, (N, K)).astype(np.float32)
    tw = Q.TiledWeight.from_float(torch.from_numpy(w).cuda(), 2)
    blocks = O.quantize_blocks(O.GGML_Q4_0, w.astype(np.float64))
    for M in (5, 96):
        xb = O.f32_array_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
        xf = O.bf16_bits_to_f32_array(xb).reshape(M, K)
        x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16).reshape(M, K)
        y = Q.weight_only_matmul(tw, x).cpu().numpy()
        ref = O.gemv_blocks(O.GGML_Q4_0, blocks, N, K, xf.astype(np.float64))
        assert rel_err(y, ref) <= 1e-3
