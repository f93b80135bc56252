/*
 * vxo.c -- CPU oracle (TEST INFRASTRUCTURE ONLY; see vxo.h).
 *
 * A plain-C restatement of the reference's CPU arithmetic for the quantized
 * inference path. The reference is Rust (no toolchain in this image), so this
 * restatement stands in for it; it is pinned against the reference's own unit
 * tests (known-answer vectors) in tests/test_oracle_kats.py.
 *
 * Build: see oracle/Makefile (-O2 -ffp-contract=off so that, like rustc, no
 * multiply-add is fused and every f32/f64 operation rounds on its own).
 */
#include "vxo.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* Rust `f64 as i64` saturates and maps NaN to 0. */
static int64_t rust_f64_to_i64(double v) {
    if (isnan(v)) return 0;
    if (v >= 9223372036854775807.0) return INT64_MAX;
    if (v <= -9223372036854775808.0) return INT64_MIN;
    return (int64_t)v;
}

static int64_t clamp_i64(int64_t v, int64_t lo, int64_t hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

static uint32_t f32_bits(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static float bits_f32(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* src/tensor_engine.rs:42-64 -- truncating f32 -> f16 (no rounding). */
uint16_t vxo_f32_to_f16(float x) {
    uint32_t bits = f32_bits(x);
    uint32_t sign = (bits >> 16) & 0x8000u;
    int32_t exp = (int32_t)((bits >> 23) & 0xFFu);
    uint32_t frac = bits & 0x7FFFFFu;
    if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (frac != 0 ? 0x200u : 0u));
    int32_t new_exp = exp - 127 + 15;
    if (new_exp >= 31) return (uint16_t)(sign | 0x7C00u);
    if (new_exp <= 0) {
        if (new_exp < -10) return (uint16_t)sign;
        uint32_t f = (frac | 0x800000u) >> (uint32_t)(1 - new_exp);
        return (uint16_t)(sign | (f >> 13));
    }
    return (uint16_t)(sign | ((uint32_t)new_exp << 10) | (frac >> 13));
}

/* src/tensor_engine.rs:66-92. Subnormals decode with exponent 127-15-e
 * (half the IEEE value) -- kept as in the reference. */
float vxo_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t frac = h & 0x3FFu;
    if (exp == 0) {
        if (frac == 0) return bits_f32(sign);
        int32_t e = 0;
        uint32_t f = frac;
        while ((f & 0x400u) == 0) { f <<= 1; e += 1; }
        uint32_t exp32 = (uint32_t)(127 - 15 - e);
        uint32_t frac32 = (f & 0x3FFu) << 13;
        return bits_f32(sign | (exp32 << 23) | frac32);
    }
    if (exp == 31) return bits_f32(sign | 0x7F800000u | (frac << 13));
    uint32_t exp32 = exp + 127 - 15;
    return bits_f32(sign | (exp32 << 23) | (frac << 13));
}

/* src/tensor_engine.rs:94-99 -- round to nearest even via bias. */
uint16_t vxo_f32_to_bf16(float x) {
    uint32_t bits = f32_bits(x);
    uint32_t bias = 0x7FFFu + ((bits >> 16) & 1u);
    return (uint16_t)((bits + bias) >> 16);
}

/* src/tensor_engine.rs:101-103 */
float vxo_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

/* src/quantize.rs:585-591. Rust's f64::max ignores NaN like C fmax. */
double vxo_calibrate_minmax(const double *data, size_t n) {
    if (n == 0) return 1.0;
    double m = 0.0;
    for (size_t i = 0; i < n; i++) m = fmax(m, fabs(data[i]));
    if (m == 0.0) return 1.0;
    return m / 127.0;
}

/* src/quantize.rs:594-600 */
double vxo_calibrate_minmax_range(const double *data, size_t n, double qmin, double qmax) {
    if (n == 0) return 1.0;
    double m = 0.0;
    for (size_t i = 0; i < n; i++) m = fmax(m, fabs(data[i]));
    if (m == 0.0) return 1.0;
    return m / fmax(fabs(qmax), fabs(qmin));
}

/* src/quantize.rs:664-672 -- low nibble = even index; odd tail pads hi with 0. */
void vxo_pack_int4(const int8_t *values, size_t n, uint8_t *out) {
    for (size_t i = 0, o = 0; i < n; i += 2, o++) {
        uint8_t lo = (uint8_t)values[i] & 0x0F;
        uint8_t hi = (i + 1 < n) ? ((uint8_t)values[i + 1] & 0x0F) : 0;
        out[o] = (uint8_t)(lo | (hi << 4));
    }
}

/* src/quantize.rs:682-687 */
static int8_t sign_extend_4bit(uint8_t v) {
    v &= 0x0F;
    return (v & 0x08) ? (int8_t)(v | 0xF0) : (int8_t)v;
}

/* src/quantize.rs:675-680 */
void vxo_unpack_int4(const uint8_t *packed, size_t nbytes, int8_t *out) {
    for (size_t i = 0; i < nbytes; i++) {
        out[2 * i] = sign_extend_4bit(packed[i] & 0x0F);
        out[2 * i + 1] = sign_extend_4bit((packed[i] >> 4) & 0x0F);
    }
}

/* src/quantize.rs:694-704 */
void vxo_pack_int2(const int8_t *values, size_t n, uint8_t *out) {
    for (size_t i = 0, o = 0; i < n; i += 4, o++) {
        uint8_t byte = 0;
        for (size_t j = 0; j < 4 && i + j < n; j++)
            byte |= (uint8_t)(((uint8_t)values[i + j] & 0x03) << (j * 2));
        out[o] = byte;
    }
}

/* src/quantize.rs:707-722 */
void vxo_unpack_int2(const uint8_t *packed, size_t nbytes, int8_t *out) {
    for (size_t i = 0; i < nbytes; i++) {
        for (int j = 0; j < 4; j++) {
            uint8_t b = (packed[i] >> (j * 2)) & 0x03;
            out[4 * i + j] = (b & 0x02) ? (int8_t)(b | 0xFC) : (int8_t)b;
        }
    }
}

size_t vxo_num_groups(size_t n, size_t group_size) {
    if (group_size == 0) return 1;
    return (n + group_size - 1) / group_size;
}

/* One quantized code, src/quantize.rs:105-108 / 148-151 / 192-195:
 * q = if scale == 0 { 0 } else { clamp(round(v/scale) as i64 + zp, qmin, qmax) } */
static int64_t quant_code(double v, double scale, int64_t zp, int64_t qmin, int64_t qmax) {
    if (scale == 0.0) return 0;
    return clamp_i64(rust_f64_to_i64(round(v / scale)) + zp, qmin, qmax);
}

/* QuantTensor::quantize for INT8/INT4/INT2 (src/quantize.rs:81-235). */
size_t vxo_quantize(const double *data, size_t n, int fmt, size_t group_size,
                    uint8_t *packed, double *scales, int64_t *zps) {
    int64_t qmin, qmax;
    double cmin, cmax;
    switch (fmt) {
    case VXO_INT8: qmin = -128; qmax = 127; cmin = 0; cmax = 0; break;
    case VXO_INT4: qmin = -8; qmax = 7; cmin = -8.0; cmax = 7.0; break;
    case VXO_INT2: qmin = -2; qmax = 1; cmin = -2.0; cmax = 1.0; break;
    default: return 0;
    }
    size_t gs = group_size ? group_size : (n ? n : 1);
    int8_t *q = (int8_t *)malloc(n ? n : 1);
    size_t g = 0;
    if (n == 0) {
        /* calibrate on an empty slice gives (1.0, 0) */
        scales[0] = 1.0; zps[0] = 0;
    }
    for (size_t s = 0; s < n; s += gs, g++) {
        size_t len = (s + gs <= n) ? gs : n - s;
        double scale = (fmt == VXO_INT8) ? vxo_calibrate_minmax(data + s, len)
                                         : vxo_calibrate_minmax_range(data + s, len, cmin, cmax);
        scales[g] = scale;
        zps[g] = 0;
        for (size_t i = 0; i < len; i++) q[s + i] = (int8_t)quant_code(data[s + i], scale, 0, qmin, qmax);
    }
    size_t nbytes;
    if (fmt == VXO_INT8) {
        for (size_t i = 0; i < n; i++) packed[i] = (uint8_t)q[i];
        nbytes = n;
    } else if (fmt == VXO_INT4) {
        vxo_pack_int4(q, n, packed);
        nbytes = (n + 1) / 2;
    } else {
        vxo_pack_int2(q, n, packed);
        nbytes = (n + 3) / 4;
    }
    free(q);
    return nbytes;
}

/* QuantTensor::dequantize_int8/int4/int2 (src/quantize.rs:325-400).
 * group_size == 0: PerTensor with scales[0]/zps[0]. */
void vxo_dequantize(const uint8_t *packed, size_t nbytes, size_t numel, int fmt,
                    size_t group_size, const double *scales, const int64_t *zps, double *out) {
    size_t ncodes;
    int8_t *codes;
    if (fmt == VXO_INT8) {
        ncodes = nbytes;
        codes = (int8_t *)malloc(ncodes ? ncodes : 1);
        for (size_t i = 0; i < nbytes; i++) codes[i] = (int8_t)packed[i];
    } else if (fmt == VXO_INT4) {
        ncodes = 2 * nbytes;
        codes = (int8_t *)malloc(ncodes ? ncodes : 1);
        vxo_unpack_int4(packed, nbytes, codes);
    } else {
        ncodes = 4 * nbytes;
        codes = (int8_t *)malloc(ncodes ? ncodes : 1);
        vxo_unpack_int2(packed, nbytes, codes);
    }
    size_t produced = 0;
    if (group_size == 0) {
        for (size_t i = 0; i < ncodes && produced < numel; i++)
            out[produced++] = (double)((int64_t)codes[i] - zps[0]) * scales[0];
    } else {
        for (size_t gi = 0, s = 0; s < ncodes; s += group_size, gi++) {
            size_t len = (s + group_size <= ncodes) ? group_size : ncodes - s;
            for (size_t i = 0; i < len; i++) {
                if (produced >= numel) break;
                out[produced++] = (double)((int64_t)codes[s + i] - zps[gi]) * scales[gi];
            }
        }
    }
    /* the reference returns a shorter Vec when data runs out; pad with 0 */
    for (; produced < numel; produced++) out[produced] = 0.0;
    free(codes);
}

/* src/quantize.rs:534-545 */
double vxo_get_scale(const double *scales, size_t n_scales, int per_group) {
    if (!per_group) return scales[0];
    if (n_scales == 0) return 1.0;
    double s = 0.0;
    for (size_t i = 0; i < n_scales; i++) s += scales[i];
    return s / (double)n_scales;
}

/* src/quantize.rs:473-515 -- i32 accumulation (wrapping), then
 * acc as f64 * a_scale * b_scale. */
void vxo_matmul_int(const uint8_t *a, const uint8_t *b, int fmt, size_t m, size_t k, size_t n,
                    double a_scale, double b_scale, int64_t a_zp, int64_t b_zp, double *out) {
    int8_t *au = NULL, *bu = NULL;
    if (fmt == VXO_INT4) {
        size_t ab = (m * k + 1) / 2, bb = (k * n + 1) / 2;
        au = (int8_t *)malloc(2 * ab + 2);
        bu = (int8_t *)malloc(2 * bb + 2);
        vxo_unpack_int4(a, ab, au);
        vxo_unpack_int4(b, bb, bu);
    }
    for (size_t i = 0; i < m; i++) {
        for (size_t j = 0; j < n; j++) {
            uint32_t acc = 0;
            for (size_t p = 0; p < k; p++) {
                int32_t av, bv;
                if (fmt == VXO_INT4) {
                    av = (int32_t)au[i * k + p] - (int32_t)a_zp;
                    bv = (int32_t)bu[p * n + j] - (int32_t)b_zp;
                } else {
                    av = (int32_t)(int8_t)a[i * k + p] - (int32_t)a_zp;
                    bv = (int32_t)(int8_t)b[p * n + j] - (int32_t)b_zp;
                }
                acc += (uint32_t)((int64_t)av * (int64_t)bv);
            }
            out[i * n + j] = (double)(int32_t)acc * a_scale * b_scale;
        }
    }
    free(au);
    free(bu);
}

/* src/quantize.rs:890-902 */
void vxo_matmul_f64(const double *a, const double *b, size_t m, size_t k, size_t n, double *out) {
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            double acc = 0.0;
            for (size_t p = 0; p < k; p++) acc += a[i * k + p] * b[p * n + j];
            out[i * n + j] = acc;
        }
}

static uint16_t rd_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* src/gguf_loader.rs:413-440 -- byte j -> elements 2j (lo), 2j+1 (hi), minus 8. */
void vxo_dequantize_q4_0(const uint8_t *data, size_t n, float *out) {
    size_t nb = (n + 31) / 32, o = 0;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *blk = data + i * 18;
        float scale = vxo_f16_to_f32(rd_u16(blk));
        for (size_t j = 0; j < 16; j++) {
            uint8_t byte = blk[2 + j];
            float lo = (float)(byte & 0x0F) - 8.0f;
            float hi = (float)((byte >> 4) & 0x0F) - 8.0f;
            size_t idx = i * 32 + j * 2;
            if (idx < n) out[o++] = lo * scale;
            if (idx + 1 < n) out[o++] = hi * scale;
        }
    }
}

/* src/gguf_loader.rs:443-472 */
void vxo_dequantize_q4_1(const uint8_t *data, size_t n, float *out) {
    size_t nb = (n + 31) / 32, o = 0;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *blk = data + i * 20;
        float scale = vxo_f16_to_f32(rd_u16(blk));
        float mn = vxo_f16_to_f32(rd_u16(blk + 2));
        for (size_t j = 0; j < 16; j++) {
            uint8_t byte = blk[4 + j];
            float lo = (float)(byte & 0x0F);
            float hi = (float)((byte >> 4) & 0x0F);
            size_t idx = i * 32 + j * 2;
            if (idx < n) out[o++] = lo * scale + mn;
            if (idx + 1 < n) out[o++] = hi * scale + mn;
        }
    }
}

/* src/gguf_loader.rs:475-498 */
void vxo_dequantize_q8_0(const uint8_t *data, size_t n, float *out) {
    size_t nb = (n + 31) / 32, o = 0;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *blk = data + i * 34;
        float scale = vxo_f16_to_f32(rd_u16(blk));
        for (size_t j = 0; j < 32; j++) {
            size_t idx = i * 32 + j;
            if (idx >= n) break;
            out[o++] = (float)(int8_t)blk[2 + j] * scale;
        }
    }
}

/* src/gguf_loader.rs:501-512; returns the number of values produced. */
size_t vxo_dequantize_f16(const uint8_t *data, size_t nbytes, size_t n, float *out) {
    size_t i = 0;
    for (; i < n; i++) {
        size_t off = i * 2;
        if (off + 1 >= nbytes) break;
        out[i] = vxo_f16_to_f32(rd_u16(data + off));
    }
    return i;
}

/* src/gguf_loader.rs:515-531 */
size_t vxo_copy_f32(const uint8_t *data, size_t nbytes, size_t n, float *out) {
    size_t i = 0;
    for (; i < n; i++) {
        size_t off = i * 4;
        if (off + 3 >= nbytes) break;
        uint32_t u = (uint32_t)data[off] | ((uint32_t)data[off + 1] << 8) |
                     ((uint32_t)data[off + 2] << 16) | ((uint32_t)data[off + 3] << 24);
        out[i] = bits_f32(u);
    }
    return i;
}

/* GGUFTensorInfo::data_size (src/gguf_loader.rs:160-166) with the block
 * sizes of GGMLQuantType (src/gguf_loader.rs:97-128). */
size_t vxo_ggml_data_size(int t, size_t n) {
    size_t bs, epb;
    switch (t) {
    case VXO_GGML_F32: bs = 4; epb = 1; break;
    case VXO_GGML_F16: bs = 2; epb = 1; break;
    case VXO_GGML_Q4_0: bs = 18; epb = 32; break;
    case VXO_GGML_Q4_1: bs = 20; epb = 32; break;
    case VXO_GGML_Q8_0: bs = 34; epb = 32; break;
    default: return 0;
    }
    return (n + epb - 1) / epb * bs;
}

/* Composed block quantizer. For each group of 32 consecutive elements of the
 * flat buffer (quantize.rs PerGroup chunking, src/quantize.rs:100-101):
 *   scale = calibrate_minmax / calibrate_minmax_range(.., -8, 7)   (585-600)
 *   code  = clamp(round(v/scale), qmin, qmax)                       (105-108, 148-151)
 * stored in the gguf_loader.rs block layout with the f64 scale narrowed
 * `as f32` then through tensor_engine::f32_to_f16 (truncating).
 * Q4_0 nibble = code + 8, i.e. byte = pack_int4(codes) ^ 0x88. A short last
 * group pads its codes with 0. */
static void quantize_blocks(const double *w, size_t n, uint8_t *blocks, int is_q4) {
    size_t nb = (n + 31) / 32;
    for (size_t b = 0; b < nb; b++) {
        size_t s = b * 32, len = (s + 32 <= n) ? 32 : n - s;
        double scale = is_q4 ? vxo_calibrate_minmax_range(w + s, len, -8.0, 7.0)
                             : vxo_calibrate_minmax(w + s, len);
        uint16_t h = vxo_f32_to_f16((float)scale);
        int8_t q[32];
        for (size_t i = 0; i < 32; i++)
            q[i] = (i < len) ? (int8_t)quant_code(w[s + i], scale, 0, is_q4 ? -8 : -128, is_q4 ? 7 : 127) : 0;
        uint8_t *blk = blocks + b * (is_q4 ? 18 : 34);
        blk[0] = (uint8_t)(h & 0xFF);
        blk[1] = (uint8_t)(h >> 8);
        if (is_q4) {
            vxo_pack_int4(q, 32, blk + 2);
            for (int j = 0; j < 16; j++) blk[2 + j] ^= 0x88;
        } else {
            for (int j = 0; j < 32; j++) blk[2 + j] = (uint8_t)q[j];
        }
    }
}

void vxo_quantize_q8_0(const double *w, size_t n, uint8_t *blocks) { quantize_blocks(w, n, blocks, 0); }
void vxo_quantize_q4_0(const double *w, size_t n, uint8_t *blocks) { quantize_blocks(w, n, blocks, 1); }

/* y = deq(W) . x per row, f64 accumulation in k order as matmul_f64
 * (src/quantize.rs:890-902) applied to weight_only_matmul(x, W^T)
 * (src/quantize.rs:845-852); dequantization per gguf_loader.rs. */
void vxo_gemv_blocks(int t, const uint8_t *blocks, size_t N, size_t K, const double *x, size_t B,
                     double *y) {
    float *row = (float *)malloc(((K + 31) / 32 * 32) * sizeof(float) + 4);
    float *all = NULL;
    size_t bpe = vxo_ggml_data_size(t, 32); /* bytes per 32-element block */
    int per_row = (K % 32 == 0);
    if (!per_row) {
        all = (float *)malloc(N * K * sizeof(float) + 4);
        if (t == VXO_GGML_Q4_0) vxo_dequantize_q4_0(blocks, N * K, all);
        else if (t == VXO_GGML_Q4_1) vxo_dequantize_q4_1(blocks, N * K, all);
        else vxo_dequantize_q8_0(blocks, N * K, all);
    }
    for (size_t r = 0; r < N; r++) {
        const float *w;
        if (per_row) {
            const uint8_t *src = blocks + r * (K / 32) * bpe;
            if (t == VXO_GGML_Q4_0) vxo_dequantize_q4_0(src, K, row);
            else if (t == VXO_GGML_Q4_1) vxo_dequantize_q4_1(src, K, row);
            else vxo_dequantize_q8_0(src, K, row);
            w = row;
        } else {
            w = all + r * K;
        }
        for (size_t b = 0; b < B; b++) {
            double acc = 0.0;
            const double *xb = x + b * K;
            for (size_t k = 0; k < K; k++) acc += xb[k] * (double)w[k];
            y[b * N + r] = acc;
        }
    }
    free(row);
    free(all);
}

/* FlashAttentionConfig::auto (src/flash_attention.rs:22-43) tile size. */
int vxo_flash_auto_tile(size_t seq_len, size_t head_dim) {
    size_t max_tile = head_dim <= 64 ? 64 : (head_dim <= 128 ? 32 : 16);
    return (int)(max_tile < seq_len ? max_tile : seq_len);
}

/* flash_attention_forward (src/flash_attention.rs:53-159), loop order kept:
 * Q tiles, KV tiles, rows, online-softmax update, dd-outer P.V update. */
void vxo_flash_attention_forward(const double *q, const double *k, const double *v, size_t n,
                                 size_t d, size_t br, size_t bc, int causal, double *out,
                                 double *lse, double *row_max) {
    double scale = 1.0 / sqrt((double)d);
    for (size_t i = 0; i < n * d; i++) out[i] = 0.0;
    for (size_t i = 0; i < n; i++) { lse[i] = -INFINITY; row_max[i] = -INFINITY; }
    if (br == 0 || bc == 0) return;
    double *m_i = (double *)malloc(br * sizeof(double));
    double *l_i = (double *)malloc(br * sizeof(double));
    double *o_i = (double *)malloc(br * d * sizeof(double));
    double *scores = (double *)malloc(bc * sizeof(double));
    double *p = (double *)malloc(bc * sizeof(double));
    for (size_t ib = 0; ib < n; ib += br) {
        size_t i_end = ib + br < n ? ib + br : n;
        size_t rows = i_end - ib;
        for (size_t ii = 0; ii < rows; ii++) {
            m_i[ii] = -INFINITY;
            l_i[ii] = 0.0;
            for (size_t dd = 0; dd < d; dd++) o_i[ii * d + dd] = 0.0;
        }
        for (size_t jb = 0; jb < n; jb += bc) {
            size_t j_end = jb + bc < n ? jb + bc : n;
            size_t cols = j_end - jb;
            if (causal && jb > i_end - 1) continue;
            for (size_t ii = 0; ii < rows; ii++) {
                size_t qi = (ib + ii) * d;
                for (size_t jj = 0; jj < cols; jj++) {
                    if (causal && (jb + jj) > (ib + ii)) { scores[jj] = -INFINITY; continue; }
                    size_t kj = (jb + jj) * d;
                    double dot = 0.0;
                    for (size_t dd = 0; dd < d; dd++) dot += q[qi + dd] * k[kj + dd];
                    scores[jj] = dot * scale;
                }
                double m_new = m_i[ii];
                for (size_t jj = 0; jj < cols; jj++) m_new = fmax(m_new, scores[jj]);
                double corr = (m_i[ii] == -INFINITY) ? 0.0 : exp(m_i[ii] - m_new);
                double l_new = l_i[ii] * corr;
                for (size_t jj = 0; jj < cols; jj++) {
                    double e = (scores[jj] == -INFINITY) ? 0.0 : exp(scores[jj] - m_new);
                    p[jj] = e;
                    l_new += e;
                }
                for (size_t dd = 0; dd < d; dd++) {
                    double o = o_i[ii * d + dd] * corr;
                    for (size_t jj = 0; jj < cols; jj++) o += p[jj] * v[(jb + jj) * d + dd];
                    o_i[ii * d + dd] = o;
                }
                m_i[ii] = m_new;
                l_i[ii] = l_new;
            }
        }
        for (size_t ii = 0; ii < rows; ii++) {
            size_t row = ib + ii;
            if (l_i[ii] > 0.0)
                for (size_t dd = 0; dd < d; dd++) out[row * d + dd] = o_i[ii * d + dd] / l_i[ii];
            row_max[row] = m_i[ii];
            lse[row] = l_i[ii] > 0.0 ? m_i[ii] + log(l_i[ii]) : -INFINITY;
        }
    }
    free(m_i); free(l_i); free(o_i); free(scores); free(p);
}

/* standard_attention (src/flash_attention.rs:163-219) */
void vxo_standard_attention(const double *q, const double *k, const double *v, size_t n, size_t d,
                            int causal, double *out) {
    double scale = 1.0 / sqrt((double)d);
    size_t nn = n * n;
    double *s = (double *)malloc((nn > 0 ? nn : 1) * sizeof(double));
    for (size_t i = 0; i < n; i++)
        for (size_t j = 0; j < n; j++) {
            if (causal && j > i) { s[i * n + j] = -INFINITY; continue; }
            double dot = 0.0;
            for (size_t dd = 0; dd < d; dd++) dot += q[i * d + dd] * k[j * d + dd];
            s[i * n + j] = dot * scale;
        }
    for (size_t i = 0; i < n; i++) {
        double mx = -INFINITY, sum = 0.0;
        for (size_t j = 0; j < n; j++) mx = fmax(mx, s[i * n + j]);
        for (size_t j = 0; j < n; j++) {
            double e = (s[i * n + j] == -INFINITY) ? 0.0 : exp(s[i * n + j] - mx);
            s[i * n + j] = e;
            sum += e;
        }
        if (sum > 0.0)
            for (size_t j = 0; j < n; j++) s[i * n + j] /= sum;
    }
    for (size_t i = 0; i < n * d; i++) out[i] = 0.0;
    for (size_t i = 0; i < n; i++)
        for (size_t j = 0; j < n; j++) {
            double w = s[i * n + j];
            for (size_t dd = 0; dd < d; dd++) out[i * d + dd] += w * v[j * d + dd];
        }
    free(s);
}

/* multi_head_flash_attention (src/flash_attention.rs:519-564): heads
 * interleaved per row ([N, H*d]); heads run serially with auto tiles. */
void vxo_multi_head_flash_attention(const double *q, const double *k, const double *v, size_t n,
                                    size_t num_heads, size_t head_dim, int causal, double *out) {
    size_t td = num_heads * head_dim;
    int tile = vxo_flash_auto_tile(n, head_dim);
    size_t sz = n * head_dim;
    if (sz == 0) sz = 1;
    double *qh = (double *)malloc(sz * sizeof(double)), *kh = (double *)malloc(sz * sizeof(double));
    double *vh = (double *)malloc(sz * sizeof(double)), *oh = (double *)malloc(sz * sizeof(double));
    double *lse = (double *)malloc((n ? n : 1) * sizeof(double));
    double *rm = (double *)malloc((n ? n : 1) * sizeof(double));
    for (size_t i = 0; i < n * td; i++) out[i] = 0.0;
    for (size_t h = 0; h < num_heads; h++) {
        for (size_t i = 0; i < n; i++)
            for (size_t dd = 0; dd < head_dim; dd++) {
                qh[i * head_dim + dd] = q[i * td + h * head_dim + dd];
                kh[i * head_dim + dd] = k[i * td + h * head_dim + dd];
                vh[i * head_dim + dd] = v[i * td + h * head_dim + dd];
            }
        vxo_flash_attention_forward(qh, kh, vh, n, head_dim, (size_t)tile, (size_t)tile, causal, oh, lse, rm);
        for (size_t i = 0; i < n; i++)
            for (size_t dd = 0; dd < head_dim; dd++)
                out[i * td + h * head_dim + dd] = oh[i * head_dim + dd];
    }
    free(qh); free(kh); free(vh); free(oh); free(lse); free(rm);
}

/* Row-sampled exact attention: the standard_attention formula
 * (src/flash_attention.rs:163-219) evaluated for the listed rows only. */
void vxo_attention_rows(const double *q, const double *k, const double *v, size_t n, size_t d,
                        int causal, const int64_t *rows, size_t nrows, double *out, double *lse) {
    double scale = 1.0 / sqrt((double)d);
    double *s = (double *)malloc((n ? n : 1) * sizeof(double));
    for (size_t r = 0; r < nrows; r++) {
        size_t i = (size_t)rows[r];
        double mx = -INFINITY, sum = 0.0;
        for (size_t j = 0; j < n; j++) {
            if (causal && j > i) { s[j] = -INFINITY; continue; }
            double dot = 0.0;
            for (size_t dd = 0; dd < d; dd++) dot += q[i * d + dd] * k[j * d + dd];
            s[j] = dot * scale;
            mx = fmax(mx, s[j]);
        }
        for (size_t j = 0; j < n; j++) {
            double e = (s[j] == -INFINITY) ? 0.0 : exp(s[j] - mx);
            s[j] = e;
            sum += e;
        }
        for (size_t dd = 0; dd < d; dd++) out[r * d + dd] = 0.0;
        for (size_t j = 0; j < n; j++) {
            double w = sum > 0.0 ? s[j] / sum : s[j];
            for (size_t dd = 0; dd < d; dd++) out[r * d + dd] += w * v[j * d + dd];
        }
        lse[r] = sum > 0.0 ? mx + log(sum) : -INFINITY;
    }
    free(s);
}

/* paged_attention (src/kv_cache.rs:95-112): keys/values are [ctx, head_dim]. */
void vxo_paged_attention(const double *query, const double *keys, const double *values, size_t ctx,
                         size_t head_dim, double *out) {
    for (size_t i = 0; i < head_dim; i++) out[i] = 0.0;
    if (ctx == 0) return;
    double scale = 1.0 / sqrt((double)head_dim);
    double *sc = (double *)malloc(ctx * sizeof(double));
    double mx = -INFINITY, sum = 0.0;
    for (size_t t = 0; t < ctx; t++) {
        double dot = -0.0;
        for (size_t i = 0; i < head_dim; i++) dot += keys[t * head_dim + i] * query[i];
        sc[t] = dot * scale;
        mx = fmax(mx, sc[t]);
    }
    for (size_t t = 0; t < ctx; t++) { sc[t] = exp(sc[t] - mx); sum += sc[t]; }
    for (size_t t = 0; t < ctx; t++) {
        double w = sc[t] / sum;
        for (size_t i = 0; i < head_dim; i++) out[i] += w * values[t * head_dim + i];
    }
    free(sc);
}

/* layer_norm (RMS form with bias), stdlib/ai/transformer.vx:413-439.
 * The .vx defines its own series sqrt/exp/log/sin/cos; libm is used here. */
void vxo_rmsnorm_bias(const double *x, const double *w, const double *b, size_t n, double eps,
                      double *out) {
    double ss = 0.0;
    for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
    double rms = sqrt(ss / (double)n + eps);
    double inv = 1.0 / rms;
    for (size_t j = 0; j < n; j++) out[j] = x[j] * inv * w[j] + b[j];
}

/* rope_embed, stdlib/ai/transformer.vx:442-466: adjacent pairs rotated by
 * theta = pos / exp(pair * ln(10000) / dim); an odd tail passes through. */
void vxo_rope_embed(const double *x, size_t n, int64_t pos, int64_t dim, double *out) {
    size_t i = 0;
    while (i < n) {
        if (i + 1 < n) {
            double pair = (double)(i / 2);
            double theta = (double)pos / exp(pair * log(10000.0) / (double)dim);
            double c = cos(theta), s = sin(theta);
            out[i] = x[i] * c - x[i + 1] * s;
            out[i + 1] = x[i] * s + x[i + 1] * c;
            i += 2;
        } else {
            out[i] = x[i];
            i += 1;
        }
    }
}

/* the `rope` builtin, src/interpreter.rs:2368-2373: pair i of x
 * (x[2i], x[2i+1]) rotated by the angle freqs[i], or by 0 for
 * i >= n_freqs; an odd tail passes through. */
void vxo_rope_builtin(const double *x, size_t n, const double *freqs, size_t n_freqs, double *out) {
    for (size_t i = 0; i < n; i++) out[i] = x[i];
    for (size_t i = 0; i < n / 2; i++) {
        double f = i < n_freqs ? freqs[i] : 0.0;
        double s = sin(f), c = cos(f);
        out[2 * i] = x[2 * i] * c - x[2 * i + 1] * s;
        out[2 * i + 1] = x[2 * i] * s + x[2 * i + 1] * c;
    }
}

/* _vec_add, stdlib/ai/transformer.vx:353-366 (the residual add). */
void vxo_vec_add(const double *a, const double *b, size_t n, double *out) {
    for (size_t i = 0; i < n; i++) out[i] = a[i] + b[i];
}

/* _silu, stdlib/ai/transformer.vx:176-182 */
double vxo_silu(double x) { return x * (1.0 / (1.0 + exp(0.0 - x))); }

/* _matvec, stdlib/ai/transformer.vx:332-350 */
void vxo_matvec(const double *w, const double *v, size_t out_dim, size_t in_dim, double *out) {
    for (size_t i = 0; i < out_dim; i++) {
        double acc = 0.0;
        for (size_t j = 0; j < in_dim; j++) acc = acc + w[i * in_dim + j] * v[j];
        out[i] = acc;
    }
}

/* src/bytecarry.rs:491-497 */
int32_t vxo_int8_dot(const int8_t *a, const int8_t *b, size_t n) {
    uint32_t acc = 0;
    for (size_t i = 0; i < n; i++) acc += (uint32_t)((int32_t)a[i] * (int32_t)b[i]);
    return (int32_t)acc;
}

/* src/bytecarry.rs:500-513 */
int32_t vxo_int4_dot(const uint8_t *a, const uint8_t *b, size_t nbytes) {
    uint32_t acc = 0;
    for (size_t i = 0; i < nbytes; i++) {
        acc += (uint32_t)((int32_t)sign_extend_4bit(a[i] & 0x0F) * (int32_t)sign_extend_4bit(b[i] & 0x0F));
        acc += (uint32_t)((int32_t)sign_extend_4bit((a[i] >> 4) & 0x0F) *
                          (int32_t)sign_extend_4bit((b[i] >> 4) & 0x0F));
    }
    return (int32_t)acc;
}

/* flash_attention_backward (src/flash_attention.rs:227-317): D_i = dO_i . O_i,
 * then K/V tiles outer, Q tiles inner, the causal skip of whole tiles and of
 * keys past the query, P = exp(s - lse_i), and the four accumulations in the
 * reference's order. */
void vxo_flash_attention_backward(const double *q, const double *k, const double *v, const double *out,
                                  const double *grad_out, const double *lse, size_t n, size_t d, size_t br,
                                  size_t bc, int causal, double *grad_q, double *grad_k, double *grad_v) {
    const double scale = 1.0 / sqrt((double)d);
    double *di = (double *)calloc(n ? n : 1, sizeof(double));
    for (size_t i = 0; i < n * d; i++) grad_q[i] = grad_k[i] = grad_v[i] = 0.0;
    for (size_t i = 0; i < n; i++)
        for (size_t dd = 0; dd < d; dd++) di[i] += grad_out[i * d + dd] * out[i * d + dd];
    for (size_t jb = 0; jb < n; jb += bc) {
        size_t je = jb + bc < n ? jb + bc : n;
        for (size_t ib = 0; ib < n; ib += br) {
            size_t ie = ib + br < n ? ib + br : n;
            if (causal && ie - 1 < jb) continue;
            for (size_t ii = 0; ii < ie - ib; ii++) {
                size_t qi = ib + ii, qo = qi * d;
                for (size_t jj = 0; jj < je - jb; jj++) {
                    size_t kj = jb + jj;
                    if (causal && kj > qi) continue;
                    size_t ko = kj * d;
                    double dot = 0.0;
                    for (size_t dd = 0; dd < d; dd++) dot += q[qo + dd] * k[ko + dd];
                    double s = dot * scale;
                    double p = exp(s - lse[qi]);
                    for (size_t dd = 0; dd < d; dd++) grad_v[ko + dd] += p * grad_out[qo + dd];
                    double dp = 0.0;
                    for (size_t dd = 0; dd < d; dd++) dp += grad_out[qo + dd] * v[ko + dd];
                    double ds = p * (dp - di[qi]) * scale;
                    for (size_t dd = 0; dd < d; dd++) grad_q[qo + dd] += ds * k[ko + dd];
                    for (size_t dd = 0; dd < d; dd++) grad_k[ko + dd] += ds * q[qo + dd];
                }
            }
        }
    }
    free(di);
}
