"""Paged KV cache + K4 decode attention on the GPU vs the CPU oracle.

Bit-exact: block tables / free-stack order (kv_cache.rs semantics), stored
bf16 values, int8 codes and f32 scales (calibrate_minmax per token and head).
Tolerance: decode attention output is bf16: max relative error (floored at
1e-3 of max|out|) <= 1e-2 against the f64 paged_attention oracle evaluated on
the exact cached values.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O
from oracle.kv_oracle import KVOracle
from tests.parity import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def KV(cuda_ok):
    from vortex_b200 import kv_cache
    return kv_cache


def bf16_tensor(a):
    bits = O.f32_array_to_bf16_bits(np.asarray(a, dtype=np.float32))
    return torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16).reshape(np.shape(a))


def bf16_values(a):
    return O.bf16_bits_to_f32_array(O.f32_array_to_bf16_bits(np.asarray(a, dtype=np.float32))).reshape(np.shape(a))


def int8_quant_row(row):
    """Per (token, head) int8: calibrate_minmax + quantize codes (quantize.rs)."""
    packed, scales, _ = O.quantize(row.astype(np.float64), O.INT8, None)
    sc32 = np.float32(scales[0])
    return packed.view(np.int8).astype(np.float64) * np.float64(sc32)


def test_block_allocation_matches_reference_semantics(KV):
    H, D, bs = 2, 64, 16
    c = KV.PagedKVCache(num_layers=2, num_heads=H, head_dim=D, block_size=bs, max_blocks=40, max_seqs=8)
    o = KVOracle(2, H, D, bs, 40)
    rng = np.random.default_rng(0)
    plan = [(0, 5, 20), (1, 5, 3), (0, 9, 17), (0, 5, 13), (1, 9, 40), (0, 2, 1)]
    for layer, seq, T in plan:
        k = rng.standard_normal((T, H, D)).astype(np.float32)
        v = rng.standard_normal((T, H, D)).astype(np.float32)
        c.append_seq(layer, seq, bf16_tensor(k), bf16_tensor(v))
        for t in range(T):
            o.append_kv(layer, seq, bf16_values(k[t]), bf16_values(v[t]))
    torch.cuda.synchronize()
    for (layer, seq) in o.tables:
        assert c.block_table(layer, seq) == o.tables[(layer, seq)]
        kk, vv = c.get_kv(layer, seq)
        ok, ov = o.get_kv(layer, seq)
        assert np.array_equal(kk.cpu().numpy(), np.array(ok))
        assert np.array_equal(vv.cpu().numpy(), np.array(ov))
    st = c.stats()
    assert st["used_blocks"] == o.used_blocks() and st["free_blocks"] == o.free_block_count()
    assert st["num_seqs"] == o.num_tables() and st["block_size"] == bs
    c.free_seq(5)
    o.free_seq(5)
    assert c.stats()["free_blocks"] == o.free_block_count()
    # the next allocation pops the most recently freed block first
    k = rng.standard_normal((1, H, D)).astype(np.float32)
    c.append_kv(0, 11, bf16_tensor(k), bf16_tensor(k))
    o.append_kv(0, 11, None, None)
    assert c.block_table(0, 11) == o.tables[(0, 11)]


def test_out_of_blocks_is_an_error(KV):
    from vortex_b200 import _native as N
    c = KV.PagedKVCache(num_layers=1, num_heads=1, head_dim=64, block_size=16, max_blocks=2, max_seqs=4)
    k = bf16_tensor(np.zeros((33, 1, 64)))
    with pytest.raises(N.VxbError) as e:
        c.append_seq(0, 1, k, k)
    assert e.value.code == N.VXB_ENOBLOCKS
    assert c.used_blocks() == 0  # the failed append was rolled back


def int8_quant_rows_np(x):
    """Vectorised restatement of the per-(token, head) int8 rule for large
    cases: scale = absmax/127 (all-zero -> 1.0), codes = round-half-away(v/scale)
    clamped, dequantized with the f32-narrowed scale."""
    x = x.astype(np.float64)
    m = np.max(np.abs(x), axis=-1, keepdims=True)
    sc = np.where(m == 0.0, 1.0, m / 127.0)
    r = x / sc
    q = np.clip(np.sign(r) * np.floor(np.abs(r) + 0.5), -128, 127)
    return q * sc.astype(np.float32).astype(np.float64)


def _fill(KV, lens, H, D, dtype, bs=16, seed=0, keep=None, vectorised=False):
    n = len(lens)
    total_blocks = sum((L + bs - 1) // bs for L in lens) + 4
    c = KV.PagedKVCache(num_layers=1, num_heads=H, head_dim=D, block_size=bs, max_blocks=total_blocks,
                        max_seqs=n + 1, kv_dtype=dtype)
    rng = np.random.default_rng(seed)
    keys, vals = {}, {}
    for i, L in enumerate(lens):
        k = rng.standard_normal((L, H, D)).astype(np.float32)
        v = rng.standard_normal((L, H, D)).astype(np.float32)
        if L:
            c.append_seq(0, 100 + i, bf16_tensor(k), bf16_tensor(v))
        if keep is not None and i not in keep:
            continue
        kb, vb = bf16_values(k), bf16_values(v)
        if dtype == KV.I8:
            if vectorised:
                kb, vb = int8_quant_rows_np(kb), int8_quant_rows_np(vb)
            else:
                kb = np.array([[int8_quant_row(kb[t, h]) for h in range(H)] for t in range(L)]).reshape(L, H, D)
                vb = np.array([[int8_quant_row(vb[t, h]) for h in range(H)] for t in range(L)]).reshape(L, H, D)
        keys[i] = kb
        vals[i] = vb
    return c, keys, vals


def _check(KV, c, keys, vals, lens, Hq, H, D, seed=1, lse_check=True):
    n = len(lens)
    G = Hq // H
    q = np.random.default_rng(seed).standard_normal((n, Hq, D)).astype(np.float32)
    qd = bf16_tensor(q)
    qv = bf16_values(q).astype(np.float64)
    lse = torch.empty((n, Hq), dtype=torch.float32, device="cuda")
    out = c.attention(0, [100 + i for i in range(n)], qd, lse=lse).float().cpu().numpy()
    lse = lse.cpu().numpy()
    ref = np.zeros((n, Hq, D))
    rows = sorted(keys)
    for i in rows:
        for j in range(Hq):
            h = j // G
            ref[i, j] = O.paged_attention(qv[i, j], keys[i][:, h].reshape(-1), vals[i][:, h].reshape(-1), D)
    for i in rows:
        assert rel_err(out[i], ref[i]) <= 1e-2, (i, lens[i], rel_err(out[i], ref[i]))
        if lens[i] == 0:
            assert np.all(out[i] == 0)
    if lse_check:
        for i in rows:
            if lens[i] == 0:
                continue
            h = np.arange(Hq) // G
            s = np.einsum("jd,tjd->jt", qv[i], keys[i][:, h]) / math.sqrt(D)
            m = s.max(axis=1)
            want = m + np.log(np.exp(s - m[:, None]).sum(axis=1))
            assert np.max(np.abs(lse[i] - want)) < 1e-3
    return out, ref


@pytest.mark.parametrize("dtype_name", ["BF16", "I8"])
@pytest.mark.parametrize("Hq,H,D", [(32, 8, 128), (4, 4, 128), (16, 1, 64), (8, 8, 64)])
def test_decode_attention_ragged(KV, dtype_name, Hq, H, D):
    dtype = getattr(KV, dtype_name)
    lens = [1, 15, 16, 17, 100, 0, 257, 1000]
    c, keys, vals = _fill(KV, lens, H, D, dtype)
    _check(KV, c, keys, vals, lens, Hq, H, D)


@pytest.mark.parametrize("dtype_name", ["BF16", "I8"])
def test_decode_attention_block_size_32(KV, dtype_name):
    """Cache blocks of 32 tokens: each block holds two 16-token pages."""
    dtype = getattr(KV, dtype_name)
    lens = [1, 31, 32, 33, 100, 0, 257]
    c, keys, vals = _fill(KV, lens, 8, 128, dtype, bs=32, seed=5)
    _check(KV, c, keys, vals, lens, 32, 8, 128)


@pytest.mark.parametrize("dtype_name", ["BF16", "I8"])
@pytest.mark.parametrize("ctx", [1024, 8192])
def test_decode_attention_c4_shapes(KV, dtype_name, ctx):
    """Decode attention config: batch 32, 32 q heads / 8 kv heads, d 128."""
    dtype = getattr(KV, dtype_name)
    lens = [ctx] * 32
    c, keys, vals = _fill(KV, lens, 8, 128, dtype, seed=ctx, keep={0, 7, 19, 31}, vectorised=True)
    _check(KV, c, keys, vals, lens, 32, 8, 128, lse_check=False)


def test_decode_attention_long_context_sampled(KV):
    """32k context for a few sequences (the oracle cost bounds the sample)."""
    lens = [32768, 32768]
    c, keys, vals = _fill(KV, lens, 8, 128, KV.BF16, seed=3)
    _check(KV, c, keys, vals, lens, 32, 8, 128, lse_check=False)


def test_append_one_token_per_sequence_then_attend(KV):
    """Decode-step pattern: each step appends one token for every sequence."""
    H, D, Hq, n = 8, 128, 32, 4
    c = KV.PagedKVCache(num_layers=1, num_heads=H, head_dim=D, block_size=16, max_blocks=64, max_seqs=8)
    rng = np.random.default_rng(9)
    keys = {i: np.zeros((0, H, D)) for i in range(n)}
    vals = {i: np.zeros((0, H, D)) for i in range(n)}
    for step in range(40):
        k = rng.standard_normal((n, H, D)).astype(np.float32)
        v = rng.standard_normal((n, H, D)).astype(np.float32)
        c.append_kv(0, [100 + i for i in range(n)], bf16_tensor(k), bf16_tensor(v))
        for i in range(n):
            keys[i] = np.concatenate([keys[i], bf16_values(k[i:i + 1])])
            vals[i] = np.concatenate([vals[i], bf16_values(v[i:i + 1])])
    _check(KV, c, keys, vals, [40] * n, Hq, H, D)


def test_decode_attention_int8_scale_range(KV):
    """int8 pages whose V magnitudes span 1e-4 .. 1e4 from token to token: the
    kernel scales P times the V scale into the f16 range per page (and
    rescales O when a page needs a smaller factor), so every page keeps its
    share of the output."""
    H, D, Hq = 8, 128, 32
    lens = [300, 77]
    c = KV.PagedKVCache(num_layers=1, num_heads=H, head_dim=D, block_size=16, max_blocks=64, max_seqs=4,
                        kv_dtype=KV.I8)
    rng = np.random.default_rng(21)
    keys, vals = {}, {}
    for i, L in enumerate(lens):
        mag = 10.0 ** rng.uniform(-4, 4, size=(L, 1, 1))
        k = (rng.standard_normal((L, H, D)) * 0.1).astype(np.float32)
        v = (rng.standard_normal((L, H, D)) * mag).astype(np.float32)
        c.append_seq(0, 100 + i, bf16_tensor(k), bf16_tensor(v))
        keys[i] = int8_quant_rows_np(bf16_values(k))
        vals[i] = int8_quant_rows_np(bf16_values(v))
    _check(KV, c, keys, vals, lens, Hq, H, D)
