"""K5 single ops through the C ABI (vxb_rmsnorm, vxb_rope, vxb_rope_angles,
vxb_swiglu, vxb_add) vs the CPU oracle's restatements of
stdlib/ai/transformer.vx:353-366, 413-466, 591-603 and the `rope` builtin
(src/interpreter.rs:2368-2373).

Tolerances: vxb_add is bit-exact (an f32 sum of two f32 values equals the f64
sum rounded to f32). RoPE rotates in f64 and rounds once to f32: max relative
error (floored at 1e-3 of max|out|) <= 1e-6. rmsnorm and swiglu write bf16:
<= 1e-2 by the same measure.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.parity import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def B(cuda_ok):
    from vortex_b200 import block_ops
    return block_ops


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


@pytest.mark.parametrize("rows,n,dim", [(1, 4096, 4096), (7, 128, 128), (3, 129, 129), (2, 1, 1), (5, 4096, 128),
                                        (1, 11, 64)])
def test_rope_embed_matches_oracle(B, rows, n, dim):
    rng = np.random.default_rng(rows * 1000 + n)
    x = rng.standard_normal((rows, n)).astype(np.float32)
    pos = np.array([0, 1, 17, 2047, 32767, 1000000, 5][:rows], dtype=np.int64)
    y = B.rope_embed(_cuda(x), pos, dim).cpu().numpy()
    for r in range(rows):
        ref = O.rope_embed(x[r].astype(np.float64), int(pos[r]), dim)
        assert rel_err(y[r], ref) <= 1e-6, (r, rel_err(y[r], ref))
        if n % 2:
            assert y[r, -1] == x[r, -1]
    if pos[0] == 0:
        assert np.array_equal(y[0], x[0])


def test_rope_embed_in_place(B):
    rng = np.random.default_rng(8)
    x = rng.standard_normal((4, 256)).astype(np.float32)
    xd = _cuda(x)
    B.rope_embed(xd, 9, 256, out=xd)
    got = xd.cpu().numpy()
    for r in range(4):
        assert rel_err(got[r], O.rope_embed(x[r].astype(np.float64), 9, 256)) <= 1e-6


@pytest.mark.parametrize("n,n_freqs", [(64, 32), (64, 10), (65, 40), (9, 0), (3, 1)])
def test_rope_builtin_matches_oracle(B, n, n_freqs):
    rng = np.random.default_rng(n + n_freqs)
    x = rng.standard_normal((3, n)).astype(np.float32)
    freqs = rng.uniform(-50, 50, n_freqs)
    y = B.rope(_cuda(x), freqs).cpu().numpy()
    for r in range(3):
        ref = O.rope_builtin(x[r].astype(np.float64), freqs)
        assert rel_err(y[r], ref) <= 1e-6
        # pairs past the frequency list turn by 0 and come back unchanged
        assert np.array_equal(y[r, 2 * n_freqs:], x[r, 2 * n_freqs:])


@pytest.mark.parametrize("n", [1, 3, 4, 1023, 4096, 32768 * 4 + 5, 1 << 24])
def test_vec_add_bit_exact(B, n):
    rng = np.random.default_rng(n)
    a = (rng.standard_normal(n) * 10.0 ** rng.uniform(-8, 8, n)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    got = B.vec_add(_cuda(a), _cuda(b)).cpu().numpy()
    if n <= 4096:
        want = O.vec_add(a, b).astype(np.float32)
    else:
        want = (a.astype(np.float64) + b.astype(np.float64)).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_vec_add_unaligned_and_in_place(B):
    rng = np.random.default_rng(2)
    a = rng.standard_normal(1001).astype(np.float32)
    b = rng.standard_normal(1001).astype(np.float32)
    ad, bd = _cuda(a), _cuda(b)
    got = B.vec_add(ad[1:], bd[:-1]).cpu().numpy()  # 4-byte offset: scalar path
    assert np.array_equal(got, (a[1:] + b[:-1]).astype(np.float32))
    B.vec_add(ad, bd, out=ad)
    assert np.array_equal(ad.cpu().numpy(), O.vec_add(a, b).astype(np.float32))


@pytest.mark.parametrize("rows,n", [(1, 4096), (3, 4096), (2, 100), (4, 11008), (1, 5)])
def test_layer_norm_matches_oracle(B, rows, n):
    rng = np.random.default_rng(rows + n)
    x = rng.standard_normal((rows, n)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    y = B.layer_norm(_cuda(x), _cuda(w), _cuda(b), 1e-5).float().cpu().numpy()
    for r in range(rows):
        ref = O.rmsnorm_bias(x[r], w, b, 1e-5)
        assert rel_err(y[r], ref) <= 1e-2


@pytest.mark.parametrize("rows,ffn", [(1, 11008), (5, 1000), (32, 11008)])
def test_swiglu_matches_oracle(B, rows, ffn):
    rng = np.random.default_rng(rows + ffn)
    gu = (rng.standard_normal((rows, 2 * ffn)) * 3).astype(np.float32)
    y = B.swiglu(_cuda(gu)).float().cpu().numpy()
    g, u = gu[:, :ffn].astype(np.float64), gu[:, ffn:].astype(np.float64)
    ref = g * (1.0 / (1.0 + np.exp(-g))) * u
    assert O.silu(1.5) == pytest.approx(1.5 / (1.0 + np.exp(-1.5)), rel=1e-15)
    for r in range(rows):
        assert rel_err(y[r], ref[r]) <= 1e-2


def test_empty_inputs_give_empty_outputs(B):
    """rope_embed / _vec_add of empty vectors are empty in the reference."""
    e = torch.zeros(0, 8, device="cuda")
    assert B.rope_embed(e, 3, 8).shape == (0, 8)
    assert B.rope(e, [0.5]).shape == (0, 8)
    z = torch.zeros(0, device="cuda")
    assert B.vec_add(z, z).numel() == 0
    assert O.rope_embed(np.zeros(0), 3, 8).size == 0 and O.vec_add([], []).size == 0


def test_bad_arguments_are_errors(B):
    from vortex_b200 import _native as N
    from vortex_b200.quant import _dptr, _stream_ptr, context
    x = torch.zeros(2, 8, device="cuda")
    p = torch.zeros(2, dtype=torch.int64, device="cuda")
    ctx = context(0)
    with pytest.raises(N.VxbError) as e:
        ctx.call("vxb_rope", _dptr(x), 2, 8, _dptr(p), 0, _dptr(x), _stream_ptr())
    assert e.value.code == N.VXB_EINVAL
    with pytest.raises(N.VxbError) as e:
        ctx.call("vxb_rope_angles", _dptr(x), 2, 8, None, 3, _dptr(x), _stream_ptr())
    assert e.value.code == N.VXB_EINVAL
    with pytest.raises(N.VxbError) as e:
        ctx.call("vxb_add", _dptr(x), None, 16, _dptr(x), _stream_ptr())
    assert e.value.code == N.VXB_EINVAL
