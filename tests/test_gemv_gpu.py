"""K1 decode GEMV on the GPU vs the CPU oracle (restated reference path).

Bit-exact: device quantizer, tiled layout round trip.
Tolerance: y = deq(W) x with f32 accumulation, max relative error (floored at
1e-3 of max|y|) <= 1e-3 for f32 output and <= 1e-2 for bf16 output.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.parity import rel_err, norm_err, bf16_round

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def Q(cuda_ok):
    from vortex_b200 import quant
    return quant


OFMT = {2: O.GGML_Q4_0, 8: O.GGML_Q8_0}


def _weights(N, K, seed, sigma=0.02):
    return np.random.default_rng(seed).normal(0.0, sigma, (N, K)).astype(np.float32)


def _act(B, K, seed, scale=1.0):
    x = (np.random.default_rng(seed + 1).standard_normal((B, K)) * scale).astype(np.float32)
    bits = O.f32_array_to_bf16_bits(x)
    return bits, O.bf16_bits_to_f32_array(bits).reshape(B, K)


def _run(Q, fmt, w, xbits, out_dtype=torch.float32):
    N, K = w.shape
    wd = torch.from_numpy(w).cuda()
    tw = Q.TiledWeight.from_float(wd, fmt)
    x = torch.from_numpy(xbits.view(np.int16)).cuda().view(torch.bfloat16).reshape(-1, K)
    y = tw.gemv(x, out_dtype=out_dtype)
    torch.cuda.synchronize()
    return tw, y.float().cpu().numpy()


@pytest.mark.parametrize("fmt", [2, 8])
@pytest.mark.parametrize("N,K", [(16, 32), (17, 96), (1000, 160), (1024, 256)])
def test_device_quantizer_and_tiling_bit_exact(Q, fmt, N, K):
    w = _weights(N, K, N + K)
    wd = torch.from_numpy(w).cuda()
    blocks = Q.quantize_blocks(wd.reshape(-1), fmt)
    want = O.quantize_blocks(OFMT[fmt], w.astype(np.float64))
    assert np.array_equal(blocks.cpu().numpy(), want)
    tw = Q.TiledWeight(blocks, fmt, N, K)
    back = tw.to_blocks()
    assert np.array_equal(back.cpu().numpy(), want)
    deq = Q.dequantize_blocks(blocks, fmt, N * K)
    assert np.array_equal(deq.cpu().numpy(), O.dequantize_blocks(OFMT[fmt], want, N * K))


@pytest.mark.parametrize("fmt", [2, 8])
@pytest.mark.parametrize("N,K", [(16, 32), (17, 96), (1000, 160), (1024, 256), (300, 4096)])
@pytest.mark.parametrize("B", [1, 2, 3, 4, 5, 8, 9, 32])
def test_gemv_small_shapes(Q, fmt, N, K, B):
    w = _weights(N, K, 7 * N + K)
    xbits, xf = _act(B, K, N)
    tw, y = _run(Q, fmt, w, xbits)
    ref = O.gemv_blocks(OFMT[fmt], O.quantize_blocks(OFMT[fmt], w.astype(np.float64)), N, K, xf.astype(np.float64))
    assert rel_err(y, ref) <= 1e-3, (rel_err(y, ref), norm_err(y, ref))


@pytest.mark.parametrize("fmt", [2, 8])
@pytest.mark.parametrize("N,K", [(4096, 4096), (11008, 4096), (4096, 11008)])
@pytest.mark.parametrize("B", [1, 4, 16])
def test_gemv_decode_sweep_shapes(Q, fmt, N, K, B):
    """The decode-shaped GEMV sweep at full size."""
    w = _weights(N, K, N * 3 + K)
    xbits, xf = _act(B, K, K)
    tw, y = _run(Q, fmt, w, xbits)
    ref = O.gemv_blocks(OFMT[fmt], O.quantize_blocks(OFMT[fmt], w.astype(np.float64)), N, K, xf.astype(np.float64))
    assert rel_err(y, ref) <= 1e-3, (rel_err(y, ref), norm_err(y, ref))


@pytest.mark.parametrize("fmt", [2, 8])
@pytest.mark.parametrize("B", [4, 32])
def test_gemv_bf16_output(Q, fmt, B):
    N, K = 4096, 4096
    w = _weights(N, K, 11)
    xbits, xf = _act(B, K, 12)
    tw, y = _run(Q, fmt, w, xbits, out_dtype=torch.bfloat16)
    ref = O.gemv_blocks(OFMT[fmt], O.quantize_blocks(OFMT[fmt], w.astype(np.float64)), N, K, xf.astype(np.float64))
    assert rel_err(y, ref) <= 1e-2
    # the bf16 result is the reference value rounded once
    assert rel_err(y, bf16_round(ref)) <= 1e-2


@pytest.mark.parametrize("fmt", [2, 8])
@pytest.mark.parametrize("B", [1, 4, 9])
def test_gemv_subnormal_scales_and_extreme_activations(Q, fmt, B):
    """Weights ~1e-4 give f16-subnormal block scales (reference decode: half
    the IEEE value); activations spanning 1e-6..1e5 exercise the per-row
    power-of-two staging."""
    N, K = 64, 512
    w = _weights(N, K, 3, sigma=1e-4)
    blocks = O.quantize_blocks(OFMT[fmt], w.astype(np.float64))
    h = blocks.reshape(-1, 18 if fmt == 2 else 34)[:, :2].copy().view(np.uint16)
    assert np.any((h & 0x7C00) == 0)
    x = np.random.default_rng(4).standard_normal((B, K)).astype(np.float32)
    x[0, : K // 2] *= 1e5
    x[min(1, B - 1), K // 2:] *= 1e-6
    x[B - 1, ::2] = 0.0
    xbits = O.f32_array_to_bf16_bits(x)
    xf = O.bf16_bits_to_f32_array(xbits).reshape(B, K)
    tw, y = _run(Q, fmt, w, xbits)
    ref = O.gemv_blocks(OFMT[fmt], blocks, N, K, xf.astype(np.float64))
    for b in range(B):
        assert rel_err(y[b], ref[b]) <= 1e-3, b


def test_gemv_rejects_bad_arguments(Q):
    from vortex_b200 import _native as N
    w = torch.zeros((16, 64), dtype=torch.float32, device="cuda")
    tw = Q.TiledWeight.from_float(w, "Q4_0")
    x = torch.zeros((33, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(N.VxbError) as e:
        tw.gemv(x)
    assert e.value.code == N.VXB_EINVAL
    with pytest.raises(N.VxbError):
        Q.TiledWeight(torch.zeros(10, dtype=torch.uint8, device="cuda"), "Q4_0", 16, 64)
