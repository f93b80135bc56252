"""QuantTensor::matmul on the device (vxb_quant_matmul) against the oracle's
restatement of matmul_int8 / matmul_int4 (src/quantize.rs:447-515): i32
accumulation that wraps on overflow, then acc as f64 * a_scale * b_scale with
the mean group scales (get_scale, 534-545). Integer work: the f64 outputs
must be bit-identical, including zero points and wrapped sums."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

OF = {"INT8": O.INT8, "INT4": O.INT4}


def _qt(rng, m, k, fmt, gs):
    from vortex_b200.quant import QuantTensor
    return QuantTensor.quantize(rng.standard_normal(m * k), (m, k), fmt, gs)


@pytest.mark.parametrize("fmt", ["INT8", "INT4"])
@pytest.mark.parametrize("m,k,n,gs", [(1, 1, 1, None), (3, 5, 7, None), (64, 64, 64, 32), (100, 257, 33, 32),
                                      (1024, 256, 1, 32), (130, 1000, 190, 16)])
def test_quant_matmul_bit_exact(cuda_ok, fmt, m, k, n, gs):
    rng = np.random.default_rng(m * 7 + k * 3 + n)
    a = _qt(rng, m, k, fmt, gs)
    b = _qt(rng, k, n, fmt, gs)
    got = a.matmul(b)
    want = O.matmul_int(a.data, b.data, OF[fmt], m, k, n, a.get_scale(), b.get_scale(), a.get_zero_point(),
                        b.get_zero_point())
    assert np.array_equal(got, want)


@pytest.mark.parametrize("fmt", ["INT8", "INT4"])
def test_quant_matmul_zero_points_and_wrapping(cuda_ok, fmt):
    """PerTensor zero points (the quantized_matmul builtin's tensors carry the
    _zero_point field) and sums far outside the i32 range, which wrap."""
    from vortex_b200.quant import QuantTensor
    m, k, n = 3, 40000, 5
    hi = 127 if fmt == "INT8" else 7
    lo = -128 if fmt == "INT8" else -8
    rng = np.random.default_rng(9)
    qa = np.where(rng.random(m * k) < 0.95, hi, lo).astype(np.int64)
    qb = np.where(rng.random(k * n) < 0.95, lo, hi).astype(np.int64)

    def pack(q):
        if fmt == "INT8":
            return (q & 0xFF).astype(np.uint8)
        q = q & 0xF
        if q.size % 2:
            q = np.append(q, 0)
        return (q[0::2] | (q[1::2] << 4)).astype(np.uint8)

    zps = ((0, 0), (3, -2), (-128, 127)) if fmt == "INT8" else ((0, 0), (3, -2), (-1000, 1000))
    for za, zb in zps:
        a = QuantTensor(pack(qa), (m, k), fmt, [0.5], [za])
        b = QuantTensor(pack(qb), (k, n), fmt, [0.25], [zb])
        got = a.matmul(b)
        want = O.matmul_int(a.data, b.data, OF[fmt], m, k, n, 0.5, 0.25, za, zb)
        assert np.array_equal(got, want), (za, zb)
    # with the last zero points the exact sums leave the i32 range
    exact = (qa.reshape(m, k) - zps[-1][0]) @ (qb.reshape(k, n) - zps[-1][1])
    assert np.all(np.abs(exact) > 2 ** 31)


def test_quant_matmul_reference_kat(cuda_ok):
    """The reference's INT4 quantized-matmul test (src/quantize.rs:948-972):
    [2,3] x [3,2] of values scaled into the INT4 range, each output within 50%
    of the f64 product (absolute below 0.01)."""
    from vortex_b200.quant import QuantTensor
    a = np.array([1.0, 2.0, 3.0, 4.0, 5.0, 6.0])
    b = np.array([7.0, 8.0, 9.0, 10.0, 11.0, 12.0])
    a_s = a / np.max(np.abs(a)) * 7.0
    b_s = b / np.max(np.abs(b)) * 7.0
    got = QuantTensor.quantize(a_s, (2, 3), "INT4", None).matmul(QuantTensor.quantize(b_s, (3, 2), "INT4", None))
    want = a_s.reshape(2, 3) @ b_s.reshape(3, 2)
    for q, f in zip(got, want.ravel()):
        err = abs(q - f) / abs(f) if abs(f) > 0.01 else abs(q - f)
        assert err < 0.5, (q, f)
