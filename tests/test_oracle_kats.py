"""Pin the CPU oracle to the reference's own known-answer tests.

Every vector here is transcribed from a reference unit test (file:line cited);
the oracle (oracle/vxo.c) must reproduce the reference's asserted results.
CPU only.
"""
import json
import math
import os
import struct

import numpy as np
import pytest

from oracle import oracle as O
from oracle import gguf_oracle as G

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def lcg_matrix(n, d, seed):
    """make_random_matrix (src/flash_attention.rs:589-599)."""
    state = seed
    out = []
    for _ in range(n * d):
        state = (state * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        out.append(float(state >> 33) / (4294967295.0 / 2.0) - 1.0)
    return np.array(out)


# ---------------- quantize.rs tests (src/quantize.rs:908-1123) ----------------

def test_int4_pack_unpack_roundtrip():  # src/quantize.rs:928-935
    vals = [0, 1, -1, 7, -8, 3, -4, 5]
    assert list(O.unpack_int4(O.pack_int4(vals))[:8]) == vals


def test_int2_pack_unpack_roundtrip():  # src/quantize.rs:938-945
    vals = [0, 1, -1, -2, 0, 1, -2, 1]
    assert list(O.unpack_int2(O.pack_int2(vals))[:8]) == vals


def test_int8_roundtrip_error():  # src/quantize.rs:913-925
    data = (np.arange(256) - 128.0) / 128.0
    packed, scales, zps = O.quantize(data, O.INT8, None)
    deq = O.dequantize(packed, 256, O.INT8, None, scales, zps)
    rmse = math.sqrt(np.mean((data - deq) ** 2))
    assert rmse / (data.max() - data.min()) < 0.01
    assert deq.size == 256


def test_per_group_lower_error_than_per_tensor():  # src/quantize.rs:1047-1065
    i = np.arange(256)
    data = ((i % 32) - 16.0) * (10.0 ** (i // 32 - 4))
    pt = O.quantize(data, O.INT8, None)
    pg = O.quantize(data, O.INT8, 32)
    e_pt = math.sqrt(np.mean((data - O.dequantize(pt[0], 256, O.INT8, None, pt[1], pt[2])) ** 2))
    e_pg = math.sqrt(np.mean((data - O.dequantize(pg[0], 256, O.INT8, 32, pg[1], pg[2])) ** 2))
    assert e_pg < e_pt


def test_int4_matmul_matches_f64():  # src/quantize.rs:948-972
    a = np.array([1.0, 2, 3, 4, 5, 6])
    b = np.array([7.0, 8, 9, 10, 11, 12])
    a_s = a / np.abs(a).max() * 7.0
    b_s = b / np.abs(b).max() * 7.0
    aq = O.quantize(a_s, O.INT4, None)
    bq = O.quantize(b_s, O.INT4, None)
    q = O.matmul_int(aq[0], bq[0], O.INT4, 2, 3, 2, O.get_scale(aq[1], False), O.get_scale(bq[1], False))
    f = O.matmul_f64(a_s, b_s, 2, 3, 2)
    for qv, fv in zip(q, f):
        rel = abs(qv - fv) / abs(fv) if abs(fv) > 0.01 else abs(qv - fv)
        assert rel < 0.5


def test_weight_only_matmul():  # src/quantize.rs:1068-1081
    w = np.arange(1.0, 10.0)
    x = np.array([0.1, 0.2, 0.3, 0.4, 0.5, 0.6])
    wq = O.quantize(w, O.INT4, None)
    w_deq = O.dequantize(wq[0], 9, O.INT4, None, wq[1], wq[2])
    q = O.matmul_f64(x, w_deq, 2, 3, 3)  # weight_only_matmul = dequantize + matmul_f64
    f = O.matmul_f64(x, w, 2, 3, 3)
    for qv, fv in zip(q, f):
        rel = abs(qv - fv) / abs(fv) if abs(fv) > 0.01 else abs(qv - fv)
        assert rel < 0.15


def test_calibration_rules():  # src/quantize.rs:585-600 (INT4 scale is absmax/8)
    assert O.calibrate_minmax([0.5, -1.27]) == 1.27 / 127.0
    assert O.calibrate_minmax_range([0.5, -1.6], -8.0, 7.0) == 1.6 / 8.0
    assert O.calibrate_minmax([0.0, 0.0]) == 1.0
    assert O.calibrate_minmax([]) == 1.0
    # +absmax rounds to 8 and clamps to 7 (quirk Q5); 0.5 rounds away from zero
    packed, scales, _ = O.quantize([1.6, -1.6, 0.1], O.INT4, 32)
    assert list(O.unpack_int4(packed)[:3]) == [7, -8, 1]


def test_matmul_int8_mean_scale():  # src/quantize.rs:473-491, 534-545 (mean of group scales)
    a = np.array([[1.0, -2.0], [3.0, 0.5]]).ravel()
    b = np.array([[0.25, 1.0], [-1.0, 2.0]]).ravel()
    aq = O.quantize(a, O.INT8, 2)
    bq = O.quantize(b, O.INT8, 2)
    sa, sb = O.get_scale(aq[1], True), O.get_scale(bq[1], True)
    assert sa == (aq[1][0] + aq[1][1]) / 2
    got = O.matmul_int(aq[0], bq[0], O.INT8, 2, 2, 2, sa, sb)
    qa = aq[0].view(np.int8).astype(np.int64).reshape(2, 2)
    qb = bq[0].view(np.int8).astype(np.int64).reshape(2, 2)
    want = (qa @ qb).astype(np.float64) * sa * sb
    assert np.array_equal(got, want.ravel())


# ---------------- gguf_loader.rs tests (src/gguf_loader.rs:761-941) ----------------

def test_dequantize_q4_0_basic():  # src/gguf_loader.rs:857-878
    blk = bytearray(18)
    blk[0], blk[1] = 0x00, 0x3C
    for i in range(2, 18):
        blk[i] = 0x88
    blk[2] = 0xA9
    r = O.dequantize_blocks(O.GGML_Q4_0, bytes(blk), 32)
    assert r.size == 32
    assert abs(r[0] - 1.0) < 1e-4 and abs(r[1] - 2.0) < 1e-4 and abs(r[2]) < 1e-4
    assert np.all(r[2:] == 0.0)


def test_dequantize_q8_0_basic():  # src/gguf_loader.rs:881-895
    blk = bytearray(34)
    blk[0], blk[1] = 0x00, 0x3C
    blk[2], blk[3] = 3, 0xFD
    r = O.dequantize_blocks(O.GGML_Q8_0, bytes(blk), 32)
    assert r.size == 32 and r[0] == 3.0 and r[1] == -3.0


def test_dequantize_f16_roundtrip():  # src/gguf_loader.rs:932-940
    r = O.dequantize_blocks(O.GGML_F16, bytes([0x00, 0x3C, 0x00, 0xBC, 0x00, 0x38]), 3)
    assert list(r) == [1.0, -1.0, 0.5]


def test_parse_header():  # src/gguf_loader.rs:826-833
    f = G.parse_gguf(G.build_gguf_bytes([], []))
    assert f["version"] == 3 and f["tensors"] == [] and f["metadata"] == {}


def test_parse_with_metadata():  # src/gguf_loader.rs:836-847
    f = G.parse_gguf(G.build_gguf_bytes([("test.key", G.U32, struct.pack("<I", 42))], []))
    assert f["metadata"]["test.key"] == (G.U32, 42)


def test_invalid_magic():  # src/gguf_loader.rs:850-854
    with pytest.raises(G.GGUFError):
        G.parse_gguf(bytes(32))


def test_roundtrip_f32():  # src/gguf_loader.rs:898-929
    vals = np.array([1.0, 2.5, -3.14, 0.0, 42.0, 1e-6, -1e6, 0.5], dtype=np.float32)
    data = G.build_gguf_bytes([], [("test_tensor", [8], 0, vals.tobytes())])
    f = G.parse_gguf(data)
    t = f["tensors"][0]
    assert t["name"] == "test_tensor" and t["dims"] == [8]
    off = f["tensor_data_offset"] + t["offset"]
    raw = data[off:off + G.tensor_nbytes(t)]
    got = O.dequantize_blocks(O.GGML_F32, raw, 8)
    assert np.array_equal(got, vals)


# ---------------- tensor_engine.rs conversions (src/tensor_engine.rs:42-103) ----------------

def test_f16_bf16_conversions():
    assert O.f32_to_f16(1.0) == 0x3C00
    assert O.f32_to_f16(-1.0) == 0xBC00
    assert O.f32_to_f16(0.5) == 0x3800
    # truncation, not rounding: 1 + 0.75 ulp(f16) stays at 1.0
    assert O.f32_to_f16(1.000732421875) == 0x3C00
    assert O.f32_to_f16(1e6) == 0x7C00
    assert O.f32_to_f16(1e-9) == 0x0000
    assert O.f16_to_f32(0x7BFF) == 65504.0
    # reference subnormal decode is half of IEEE (quirk kept)
    assert O.f16_to_f32(0x0001) == 2.0 ** -25
    assert O.f16_to_f32(0x0200) == 2.0 ** -16
    assert O.f32_to_bf16(1.0) == 0x3F80
    # round to nearest even at the tie
    assert O.f32_to_bf16(struct.unpack("<f", struct.pack("<I", 0x3F808000))[0]) == 0x3F80
    assert O.f32_to_bf16(struct.unpack("<f", struct.pack("<I", 0x3F818000))[0]) == 0x3F82
    x = np.random.default_rng(0).standard_normal(1000).astype(np.float32)
    assert np.array_equal(O.f32_array_to_bf16_bits(x), np.array([O.f32_to_bf16(v) for v in x], dtype=np.uint16))


# ---------------- bytecarry.rs int dots (src/bytecarry.rs:801-840) ----------------

def test_int_dots():
    assert O.int8_dot([1, -2, 3, -4], [5, 6, -7, 8]) == -60
    a = [127, -128, 64, -64, 1, -1, 0, 100]
    b = [-1, 2, -3, 4, -5, 6, -7, 8]
    assert O.int8_dot(a, b) == int(sum(x * y for x, y in zip(a, b)))
    assert O.int4_dot([0xE3], [0x41]) == -5
    assert O.int4_dot([0x32, 0x5F], [0xE1, 0xD4]) == -23


# ---------------- flash_attention.rs tests (src/flash_attention.rs:600-780, 936-954) ----------------

@pytest.mark.parametrize("n,d,seeds,tile,tol", [
    (8, 4, (42, 123, 456), 4, 1e-10),
    (32, 16, (7, 8, 9), 8, 1e-9),
])
def test_flash_matches_standard(n, d, seeds, tile, tol):
    q, k, v = (lcg_matrix(n, d, s) for s in seeds)
    out, _, _ = O.flash_attention_forward(q, k, v, d, tile, tile, False)
    ref = O.standard_attention(q, k, v, d, False)
    assert np.max(np.abs(out - ref)) < tol


def test_causal_mask():  # src/flash_attention.rs:663-700
    n, d = 8, 4
    q, k, v = (lcg_matrix(n, d, s) for s in (100, 200, 300))
    out, lse, _ = O.flash_attention_forward(q, k, v, d, 4, 4, True)
    ref = O.standard_attention(q, k, v, d, True)
    assert np.max(np.abs(out - ref)) < 1e-10
    assert np.max(np.abs(out[:d] - v[:d])) < 1e-10
    assert np.all(np.isfinite(lse))


def test_different_tile_sizes():  # src/flash_attention.rs:703-735
    n, d = 16, 8
    q, k, v = (lcg_matrix(n, d, s) for s in (55, 66, 77))
    ref = O.standard_attention(q, k, v, d, False)
    for br, bc in [(2, 2), (4, 4), (8, 8), (4, 8), (8, 4), (16, 16)]:
        out, _, _ = O.flash_attention_forward(q, k, v, d, br, bc, False)
        assert np.max(np.abs(out - ref)) < 1e-9


def test_multi_head_shape():  # src/flash_attention.rs:738-780
    n, h, hd = 8, 4, 4
    q, k, v = (lcg_matrix(n, h * hd, s) for s in (10, 20, 30))
    out = O.multi_head_flash_attention(q, k, v, h, hd, False)
    assert out.size == n * h * hd
    q3, k3, v3, o3 = (a.reshape(n, h, hd) for a in (q, k, v, out))
    for hh in range(h):
        ref = O.standard_attention(q3[:, hh].copy(), k3[:, hh].copy(), v3[:, hh].copy(), hd, False)
        assert np.max(np.abs(o3[:, hh].ravel() - ref)) < 1e-9


def test_auto_config():  # src/flash_attention.rs:936-954
    assert O.flash_auto_tile(512, 64) == 64
    assert O.flash_auto_tile(4, 64) == 4
    assert O.flash_auto_tile(512, 256) <= 16


def test_attention_rows_matches_flash():
    n, d = 24, 8
    q, k, v = (lcg_matrix(n, d, s) for s in (1, 2, 3))
    out, lse, _ = O.flash_attention_forward(q, k, v, d, 8, 8, True)
    rows = np.array([0, 5, 23])
    o2, l2 = O.attention_rows(q, k, v, d, True, rows)
    assert np.max(np.abs(o2 - out.reshape(n, d)[rows])) < 1e-12
    assert np.max(np.abs(l2 - lse[rows])) < 1e-12


# ---------------- kv_cache.rs (src/kv_cache.rs:320-415) ----------------

def test_paged_attention():  # src/kv_cache.rs:345-353
    out = O.paged_attention([1.0, 0.0], [[1.0, 0.0], [0.0, 1.0]], [[10.0, 20.0], [30.0, 40.0]], 2)
    assert out.size == 2 and out[0] > 10.0
    assert np.array_equal(O.paged_attention([1.0, 0.0], np.zeros((0, 2)), np.zeros((0, 2)), 2), [0.0, 0.0])


# ---------------- composed block quantizer ----------------

def test_composed_q4_0_matches_reference_pieces():
    rng = np.random.default_rng(5)
    w = rng.normal(0, 0.02, 96)
    blocks = O.quantize_blocks(O.GGML_Q4_0, w)
    assert blocks.size == 3 * 18
    packed, scales, _ = O.quantize(w, O.INT4, 32)  # quantize.rs PerGroup INT4 codes
    for b in range(3):
        blk = blocks[b * 18:(b + 1) * 18]
        h = int(blk[0]) | (int(blk[1]) << 8)
        assert h == O.f32_to_f16(float(np.float32(scales[b])))
        assert np.array_equal(blk[2:], packed[b * 16:(b + 1) * 16] ^ 0x88)
    deq = O.dequantize_blocks(O.GGML_Q4_0, blocks, 96)
    codes = O.unpack_int4(packed)[:96].astype(np.float32)
    sc = np.repeat(O.f16_bits_to_f32_array(blocks.reshape(3, 18)[:, :2].copy().view(np.uint16).ravel()), 32)
    assert np.array_equal(deq, codes * sc)


def test_composed_q8_0_matches_reference_pieces():
    rng = np.random.default_rng(6)
    w = rng.normal(0, 0.02, 64)
    blocks = O.quantize_blocks(O.GGML_Q8_0, w)
    packed, scales, _ = O.quantize(w, O.INT8, 32)
    for b in range(2):
        blk = blocks[b * 34:(b + 1) * 34]
        assert (int(blk[0]) | (int(blk[1]) << 8)) == O.f32_to_f16(float(np.float32(scales[b])))
        assert np.array_equal(blk[2:], packed[b * 32:(b + 1) * 32])


def test_gemv_blocks_matches_dequant_matmul():
    rng = np.random.default_rng(7)
    N, K, B = 8, 64, 3
    w = rng.normal(0, 0.02, (N, K))
    x = rng.standard_normal((B, K))
    for t in (O.GGML_Q4_0, O.GGML_Q8_0):
        bl = O.quantize_blocks(t, w)
        deq = O.dequantize_blocks(t, bl, N * K).astype(np.float64).reshape(N, K)
        y = O.gemv_blocks(t, bl, N, K, x)
        assert np.allclose(y, x @ deq.T, rtol=1e-12, atol=1e-14)


def test_golden_kats_file_matches_oracle():
    """tests/golden/reference_kats.json: vectors transcribed from reference tests."""
    with open(os.path.join(GOLDEN, "reference_kats.json")) as f:
        kats = json.load(f)
    for case in kats["int4_pack"]:
        assert list(O.pack_int4(case["values"])) == case["packed"]
    for case in kats["q4_0_block"]:
        assert list(O.dequantize_blocks(O.GGML_Q4_0, bytes(case["block"]), 32)) == case["values"]
    for case in kats["q8_0_block"]:
        assert list(O.dequantize_blocks(O.GGML_Q8_0, bytes(case["block"]), 32)) == case["values"]
    for case in kats["f16"]:
        assert O.f16_to_f32(case["bits"]) == case["value"]


# ---- f32 model, src/transformer.rs tests (1094-1250) ----

def test_tf_matmul_kat():
    # [2,3] x [3,2] -> [[4, 2], [10, 5]] (test_matmul); the oracle's linear
    # takes the weight [out, in], i.e. the transposed right factor
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[1, 0], [0, 1], [1, 0]], np.float32)
    assert np.array_equal(O.tf_linear(a, b.T), np.array([[4, 2], [10, 5]], np.float32))


def test_tf_positional_encoding_kat():
    pe = O.tf_pos_encoding(10, 8)  # test_positional_encoding
    assert pe.shape == (10, 8)
    assert abs(pe[0, 0]) < 1e-5 and abs(pe[0, 1] - 1.0) < 1e-5
    assert np.all(pe >= -1 - 1e-6) and np.all(pe <= 1 + 1e-6)


def test_rope_and_add_kats():
    # position 0 turns every pair by 0 (stdlib/ai/tensor_ops.vx:1007-1014)
    x = np.array([1.0, 0.0, 1.0, 0.0, 3.0])
    assert np.array_equal(O.rope_embed(x, 0, 4), x)
    # pair 0 at position 1 turns by exactly 1 radian, pair 1 by 1/10000^(1/4) (dim 4)
    y = O.rope_embed(np.array([1.0, 0.0, 1.0, 0.0]), 1, 4)
    assert np.allclose(y, [np.cos(1.0), np.sin(1.0), np.cos(0.1), np.sin(0.1)], rtol=0, atol=1e-15)
    # the builtin turns pair i by freqs[i] and leaves pairs past the list alone
    z = O.rope_builtin(np.array([1.0, 0.0, 2.0, 5.0, 7.0]), np.array([np.pi / 2]))
    assert np.allclose(z, [0.0, 1.0, 2.0, 5.0, 7.0], rtol=0, atol=1e-15)
    assert np.array_equal(O.vec_add([1.0, -2.5], [0.5, 2.5]), [1.5, 0.0])


def test_tf_layer_norm_kat():
    x = np.array([[1, 2, 3, 4], [5, 6, 7, 8]], np.float32)  # test_layer_norm
    y = O.tf_layernorm(x, np.ones(4, np.float32), np.zeros(4, np.float32))
    assert np.all(np.abs(y.sum(axis=1) / 4) < 1e-4)


def test_tf_softmax_and_gelu_kats():
    s = O.tf_softmax_rows(np.array([[1, 2, 3, 4]], np.float32))[0]  # test_softmax
    assert abs(s.sum() - 1) < 1e-5 and s[0] < s[1] < s[2] < s[3]
    g = O.tf_gelu(np.array([-2, -1, 0, 1, 2], np.float32))  # test_gelu_activation
    assert abs(g[2]) < 1e-5 and g[3] > 0 and g[4] > 0 and g[0] < 0


def test_tf_model_shapes_kat():
    # small_config = TransformerConfig::new(64, 16, 2, 1, 32, 32, 0.0):
    # test_model_creation / test_forward_pass_shape
    c = O.tf_config(64, 16, 2, 1, 32, 32)
    p = O.tf_init(c)
    emb, layer, final, out = 64 * 16, 4 * (16 * 16 + 16) + (32 * 16 + 32) + (16 * 32 + 16) + 4 * 16, 2 * 16, 64 * 16 + 64
    assert p.size == emb + layer + final + out
    logits = O.tf_forward(c, p, [0, 1, 2, 3])
    assert logits.shape == (4, 64) and np.all(np.isfinite(logits))
    # Xavier bound of the embedding (fan_in 64, fan_out 16) and zero biases
    assert np.max(np.abs(p[:emb])) <= np.sqrt(6 / 80) + 1e-7
    assert np.all(p[emb + 16 * 16:emb + 16 * 16 + 16] == 0)


@pytest.mark.parametrize("causal", [False, True])
def test_flash_backward_numerical_gradient(causal):  # src/flash_attention.rs:783-880
    """The oracle's flash_attention_backward against central differences of
    the forward (N=4, d=4, tiles 2, seeds 1/2/3, loss = sum of the outputs,
    eps 1e-5, |analytical - numerical| < 1e-4), as the reference's own test;
    the causal case is checked the same way."""
    n, d, eps = 4, 4, 1e-5
    q, k, v = (lcg_matrix(n, d, s) for s in (1, 2, 3))
    out, lse, _ = O.flash_attention_forward(q, k, v, d, 2, 2, causal)
    gq, gk, gv = O.flash_attention_backward(q, k, v, out, np.ones(n * d), lse, d, 2, 2, causal)
    for which, g in ((0, gq), (1, gk), (2, gv)):
        for idx in range(n * d):
            args_p = [np.array(t, dtype=np.float64) for t in (q, k, v)]
            args_m = [np.array(t, dtype=np.float64) for t in (q, k, v)]
            args_p[which][idx] += eps
            args_m[which][idx] -= eps
            lp = O.flash_attention_forward(*args_p, d, 2, 2, causal)[0].sum()
            lm = O.flash_attention_forward(*args_m, d, 2, 2, causal)[0].sum()
            assert abs(g[idx] - (lp - lm) / (2 * eps)) < 1e-4, (which, idx)
