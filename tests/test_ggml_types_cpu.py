"""GGUF tensor types beyond the kernels' tiled formats (a8): the host codec's
Q4_1 / F16 / F32 dequantization is bit-identical with the oracle's
restatement of dequantize_q4_1 / dequantize_f16 / copy_f32
(src/gguf_loader.rs:443-531), including subnormal f16 scales (the
reference's half-value subnormal decode, src/tensor_engine.rs:66-92)."""
import numpy as np
import pytest

from oracle import oracle as O


def q4_1_blocks(rng, n_blocks, subnormal=False):
    """Random Q4_1 blocks: f16 d, f16 m, 16 nibble bytes."""
    b = rng.integers(0, 256, size=(n_blocks, 20), dtype=np.uint8)
    d = (np.abs(rng.standard_normal(n_blocks)) * 0.01).astype(np.float16)
    m = (rng.standard_normal(n_blocks) * 0.05).astype(np.float16)
    if subnormal:
        d[::3] = np.float16(3e-6)  # subnormal in f16
        m[1::4] = np.float16(-2e-7)
    b[:, 0:2] = d.view(np.uint8).reshape(n_blocks, 2)
    b[:, 2:4] = m.view(np.uint8).reshape(n_blocks, 2)
    return b.ravel()


def _same_bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("subnormal", [False, True])
def test_q4_1_unpack_matches_oracle(subnormal):
    from vortex_b200 import _native as N
    from vortex_b200 import quant as Q
    rng = np.random.default_rng(41)
    blocks = q4_1_blocks(rng, 64, subnormal)
    n = 64 * 32 - 5  # a ragged tail
    got = Q.unpack_blocks(N.Q4_1, blocks, n)
    assert _same_bits(got, O.dequantize_blocks(O.GGML_Q4_1, blocks, n))


def test_f16_and_f32_unpack_match_oracle():
    from vortex_b200 import _native as N
    from vortex_b200 import quant as Q
    rng = np.random.default_rng(16)
    h = rng.integers(0, 0x7C00, size=4096, dtype=np.uint16)  # finite, subnormals included
    h[::2] |= 0x8000
    raw = h.view(np.uint8)
    assert _same_bits(Q.unpack_blocks(N.GGML_F16, raw, h.size), O.dequantize_blocks(O.GGML_F16, raw, h.size))
    f = rng.standard_normal(1000).astype(np.float32)
    assert _same_bits(Q.unpack_blocks(N.GGML_F32, f.view(np.uint8), f.size), f)


def test_block_sizes():
    from vortex_b200 import _native as N
    L = N.lib()
    assert L.vxb_block_bytes(N.Q4_1, 64) == 40 and L.vxb_block_bytes(N.Q4_1, 33) == 40
    assert L.vxb_block_bytes(N.GGML_F16, 7) == 14 and L.vxb_block_bytes(N.GGML_F32, 7) == 28
