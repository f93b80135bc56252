"""QuantTensor host side (INT8 / INT4): the product's quantizer, get_scale and
dequantize against the oracle's restatement of src/quantize.rs:81-163,
325-370, 534-545 and 585-600 - codes, scales and values bit-exact."""
import numpy as np
import pytest

from oracle import oracle as O


@pytest.mark.parametrize("fmt,ofmt", [("INT8", O.INT8), ("INT4", O.INT4)])
@pytest.mark.parametrize("n,gs", [(0, None), (1, None), (7, None), (1000, None), (1000, 32), (1001, 32),
                                  (65, 64), (96, 7)])
def test_quantize_matches_oracle(fmt, ofmt, n, gs):
    from vortex_b200.quant import QuantTensor
    rng = np.random.default_rng(n + (gs or 0))
    x = rng.standard_normal(n) * 3.0
    if n > 10:
        x[5] = 0.0
        x[7:9] = np.array([1e-300, -2.5])
    qt = QuantTensor.quantize(x, (n,), fmt, gs)
    packed, scales, zps = O.quantize(x, ofmt, gs)
    assert np.array_equal(qt.data, packed)
    assert np.array_equal(qt.scales, scales)
    assert np.array_equal(qt.zero_points, zps)
    assert qt.get_scale() == O.get_scale(scales, gs is not None)
    if n:
        assert np.array_equal(qt.dequantize(), O.dequantize(packed, n, ofmt, gs, scales, zps))


def test_all_zero_group_scale_is_one():
    from vortex_b200.quant import QuantTensor
    x = np.concatenate([np.zeros(32), np.ones(32)])
    qt = QuantTensor.quantize(x, (64,), "INT8", 32)
    assert qt.scales[0] == 1.0 and qt.scales[1] == 1.0 / 127.0
    assert np.all(qt.data[:32] == 0)
