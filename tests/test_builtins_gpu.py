"""The builtin adapters on the device against the oracle (a15).

kv_cache_attention is paged_attention over one head_dim vector per cached
token (src/kv_cache.rs:207-218, 95-112): the device cache holds one KV head
and the attention runs with one query head, scale 1/sqrt(head_dim); keys and
values are stored in bf16, so the gate is the floored relative error <= 1e-2
against the oracle on the bf16-rounded inputs. The block accounting (stats,
memory, free_seq, out-of-blocks error) follows src/kv_cache.rs:41-93.
quantized_matmul is bit-exact (integer path); flash_attention is the
builtin_flash_attention adapter over the device kernel."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.parity import bf16_round, rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("hd", [64, 128])
def test_kv_cache_builtins_one_head(cuda_ok, hd):
    from vortex_b200 import builtins as B
    cid = B.kv_cache_new(2, 8, hd, 4, 16) if hd != 64 else B.kv_cache_new(2, 8)
    bs = 4 if hd != 64 else 16
    rng = np.random.default_rng(hd)
    keys, vals = {}, {}
    for step in range(11):
        for seq in (5, 9):
            if seq == 9 and step > 6:
                continue
            k, v = rng.standard_normal(hd), rng.standard_normal(hd)
            assert B.kv_cache_append(cid, 1, seq, list(k), list(v)) is True
            keys.setdefault(seq, []).append(bf16_round(k).astype(np.float64))
            vals.setdefault(seq, []).append(bf16_round(v).astype(np.float64))
    for seq in (5, 9):
        q = rng.standard_normal(hd)
        got = np.array(B.kv_cache_attention(cid, list(q), 1, seq))
        want = O.paged_attention(bf16_round(q).astype(np.float64), np.array(keys[seq]).ravel(),
                                 np.array(vals[seq]).ravel(), hd)
        assert got.shape == (hd,)
        assert rel_err(got, want) <= 1e-2, (seq, rel_err(got, want))
    # an unknown sequence (or another layer) has no keys: zeros
    assert B.kv_cache_attention(cid, [1.0] * hd, 0, 5) == [0.0] * hd
    st = B.kv_cache_stats(cid)
    used = -(-11 // bs) + -(-7 // bs)
    assert st == {"used_blocks": used, "free_blocks": 16 - used if hd != 64 else 256 - used, "block_size": bs,
                  "num_seqs": 2}
    assert B.kv_cache_memory(cid) == used * bs * hd * 2 * 8
    assert B.kv_cache_free_seq(cid, 9) is True
    assert B.kv_cache_stats(cid)["used_blocks"] == -(-11 // bs)


def test_kv_cache_builtin_errors(cuda_ok):
    from vortex_b200 import builtins as B
    cid = B.kv_cache_new(1, 1, 64, 2, 2)
    for t in range(4):
        B.kv_cache_append(cid, 0, 0, [0.5] * 64, [1.0] * 64)
    with pytest.raises(B.BuiltinError, match="KV cache out of blocks"):
        B.kv_cache_append(cid, 0, 0, [0.5] * 64, [1.0] * 64)
    with pytest.raises(B.BuiltinError, match="KV cache out of blocks"):
        B.kv_cache_append(cid, 0, 7, [0.5] * 64, [1.0] * 64)
    # the failed append of a new sequence leaves its (empty) table, as the reference
    assert B.kv_cache_stats(cid) == {"used_blocks": 2, "free_blocks": 0, "block_size": 2, "num_seqs": 2}
    B.kv_cache_free_seq(cid, 0)
    assert B.kv_cache_stats(cid)["used_blocks"] == 0
    assert B.kv_cache_append(cid, 0, 7, [0.5] * 64, [1.0] * 64) is True
    with pytest.raises(B.BuiltinError, match="invalid cache"):
        B.kv_cache_stats(cid + 1000)
    with pytest.raises(B.BuiltinError, match="need cache_id"):
        B.kv_cache_append(None, 0, 0, [0.0], [0.0])
    with pytest.raises(B.BuiltinError, match="need key"):
        B.kv_cache_append(cid, 0, 0)


@pytest.mark.parametrize("fmt", ["INT8", "INT4"])
def test_quantized_matmul_builtin(cuda_ok, fmt):
    from vortex_b200 import builtins as B
    rng = np.random.default_rng(4)
    a = B.quantize(list(rng.standard_normal(6 * 40)), [6, 40], fmt, 32)
    b = B.quantize(list(rng.standard_normal(40 * 5)), [40, 5], fmt, 32)
    got = B.quantized_matmul(a, b)
    ofmt = O.INT8 if fmt == "INT8" else O.INT4
    want = O.matmul_int(np.array(a["_data"], np.uint8), np.array(b["_data"], np.uint8), ofmt, 6, 40, 5,
                        a["_scale"], b["_scale"], 0, 0)
    assert got == list(want)


def test_flash_attention_builtin(cuda_ok):
    from vortex_b200 import builtins as B
    rng = np.random.default_rng(8)
    n, H = 40, 2
    q, k, v = (bf16_round(rng.standard_normal((n, H * 128))).astype(np.float64) for _ in range(3))
    got = np.array(B.flash_attention(q.tolist(), k.tolist(), v.tolist(), H, True))
    want = O.multi_head_flash_attention(q, k, v, H, 128, True).reshape(n, H * 128)
    assert rel_err(got, want) <= 1e-2
    assert B.flash_attention([], [], []) == []
    with pytest.raises(B.BuiltinError, match="not divisible by 3 heads"):
        B.flash_attention(q.tolist(), k.tolist(), v.tolist(), 3, True)
