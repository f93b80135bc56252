/* CPU oracle (test infrastructure only): restatement in C of the reference's
 * f32 GPT-style model, src/transformer.rs:15-841 (SimpleRng, Linear,
 * LayerNorm, MultiHeadAttention, FeedForward, TransformerLayer, sinusoidal
 * positional encoding, TransformerModel::new / forward). Every loop keeps the
 * reference's order and every operation is a separately rounded f32
 * operation (built with -ffp-contract=off); exp/tanh/sqrt/sin/cos/pow are the
 * C library's, as Rust's f32 methods on Linux. */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "vxo.h"

/* SimpleRng: xorshift64 seeded with seed + 1 (src/transformer.rs:15-45) */
typedef struct {
    uint64_t s;
} tf_rng;

static uint64_t tf_next_u64(tf_rng *r) {
    r->s ^= r->s << 13;
    r->s ^= r->s >> 7;
    r->s ^= r->s << 17;
    return r->s;
}

static float tf_next_f32(tf_rng *r) {
    const uint64_t v = tf_next_u64(r);
    const float u = (float)(v >> 40) / (float)(1ull << 24);
    return u * 2.0f - 1.0f;
}

static float tf_xavier(tf_rng *r, size_t fan_in, size_t fan_out) {
    const float limit = sqrtf(6.0f / (float)(fan_in + fan_out));
    return tf_next_f32(r) * limit;
}

/* params_vec layout (src/transformer.rs:806-815 and the per-module
 * params_vec): embedding [vocab, d]; per layer: wq, wk, wv, wo (weight
 * [out, in] then bias [out]), linear1 (d -> d_ff), linear2 (d_ff -> d),
 * norm1 gamma, beta, norm2 gamma, beta; final_norm gamma, beta; output
 * projection weight [vocab, d] and bias [vocab]. */
static size_t tf_layer_params(const vxo_tf_config *c) {
    const size_t d = c->d_model, f = c->d_ff;
    return 4 * (d * d + d) + (f * d + f) + (d * f + d) + 4 * d;
}

size_t vxo_tf_param_count(const vxo_tf_config *c) {
    return c->vocab * c->d_model + c->n_layers * tf_layer_params(c) + 2 * c->d_model + c->vocab * c->d_model +
           c->vocab;
}

static void tf_linear_init(tf_rng *r, size_t in, size_t out, float *p) {
    for (size_t i = 0; i < out * in; i++) p[i] = tf_xavier(r, in, out);
    for (size_t i = 0; i < out; i++) p[out * in + i] = 0.0f;
}

/* TransformerModel::new (src/transformer.rs:679-721): the generator is drawn
 * in creation order (embedding, then per layer wq wk wv wo linear1 linear2,
 * then the output projection); norms are gamma 1, beta 0. */
void vxo_tf_init(const vxo_tf_config *c, uint64_t seed, float *p) {
    tf_rng r = {seed + 1};
    const size_t d = c->d_model, f = c->d_ff, V = c->vocab;
    for (size_t i = 0; i < V * d; i++) p[i] = tf_xavier(&r, V, d);
    p += V * d;
    for (size_t l = 0; l < c->n_layers; l++) {
        for (int m = 0; m < 4; m++) {
            tf_linear_init(&r, d, d, p);
            p += d * d + d;
        }
        tf_linear_init(&r, d, f, p);
        p += f * d + f;
        tf_linear_init(&r, f, d, p);
        p += d * f + d;
        for (int m = 0; m < 2; m++) {
            for (size_t i = 0; i < d; i++) p[i] = 1.0f;
            for (size_t i = 0; i < d; i++) p[d + i] = 0.0f;
            p += 2 * d;
        }
    }
    for (size_t i = 0; i < d; i++) p[i] = 1.0f;
    for (size_t i = 0; i < d; i++) p[d + i] = 0.0f;
    p += 2 * d;
    tf_linear_init(&r, d, V, p);
}

/* make_pos_encoding (src/transformer.rs:655-670) */
void vxo_tf_pos_encoding(size_t max_len, size_t d, float *out) {
    for (size_t pos = 0; pos < max_len; pos++)
        for (size_t i = 0; i < d; i++) {
            const float angle = (float)pos / powf(10000.0f, (float)(2 * (i / 2)) / (float)d);
            out[pos * d + i] = (i % 2 == 0) ? sinf(angle) : cosf(angle);
        }
}

/* Linear::forward (src/transformer.rs:332-352): input @ weight^T (the
 * transposed copy's matmul sums over the input features in order), then the
 * bias in a separate add. */
void vxo_tf_linear(const float *x, size_t m, const float *w, const float *b, size_t in, size_t out, float *y) {
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < out; j++) {
            float sum = 0.0f;
            for (size_t p = 0; p < in; p++) sum += x[i * in + p] * w[j * in + p];
            y[i * out + j] = sum;
        }
    if (b)
        for (size_t i = 0; i < m; i++)
            for (size_t j = 0; j < out; j++) y[i * out + j] = y[i * out + j] + b[j];
}

/* LayerNorm::forward (src/transformer.rs:405-428) */
void vxo_tf_layernorm(const float *x, size_t rows, size_t d, const float *g, const float *b, float eps, float *y) {
    for (size_t i = 0; i < rows; i++) {
        const float *row = x + i * d;
        float s = 0.0f;
        for (size_t j = 0; j < d; j++) s += row[j];
        const float mean = s / (float)d;
        float v = 0.0f;
        for (size_t j = 0; j < d; j++) v += (row[j] - mean) * (row[j] - mean);
        const float var = v / (float)d;
        const float std_inv = 1.0f / sqrtf(var + eps);
        for (size_t j = 0; j < d; j++) y[i * d + j] = (row[j] - mean) * std_inv * g[j] + b[j];
    }
}

/* gelu (src/transformer.rs:245-254), tanh form */
void vxo_tf_gelu(const float *x, size_t n, float *y) {
    const float sqrt_2_pi = sqrtf(2.0f / 3.14159265358979323846f);
    for (size_t i = 0; i < n; i++) {
        const float v = x[i];
        const float inner = sqrt_2_pi * (v + 0.044715f * v * v * v);
        y[i] = 0.5f * v * (1.0f + tanhf(inner));
    }
}

/* softmax_2d (src/transformer.rs:194-218) */
void vxo_tf_softmax_rows(const float *x, size_t rows, size_t cols, float *y) {
    for (size_t i = 0; i < rows; i++) {
        const float *row = x + i * cols;
        float mx = -INFINITY;
        for (size_t j = 0; j < cols; j++) mx = fmaxf(mx, row[j]);
        float sum = 0.0f;
        for (size_t j = 0; j < cols; j++) {
            const float v = expf(row[j] - mx);
            y[i * cols + j] = v;
            sum += v;
        }
        if (sum > 0.0f)
            for (size_t j = 0; j < cols; j++) y[i * cols + j] /= sum;
    }
}

/* MultiHeadAttention::forward with q = k = v input (src/transformer.rs:
 * 510-567): per-head projections, scores = (Q K^T) * (1/sqrt(hd)), mask
 * entries < 0.5 -> -1e9 (mask [S, S] broadcast over heads), softmax, P V,
 * heads merged, output projection. */
static void tf_mha(const float *p, const float *x, size_t S, size_t d, size_t H, const float *mask, float *out,
                   float *scratch) {
    const size_t hd = d / H;
    float *q = scratch, *k = q + S * d, *v = k + S * d, *sc = v + S * d, *pr = sc + S * S, *merged = pr + S * S;
    vxo_tf_linear(x, S, p, p + d * d, d, d, q);
    p += d * d + d;
    vxo_tf_linear(x, S, p, p + d * d, d, d, k);
    p += d * d + d;
    vxo_tf_linear(x, S, p, p + d * d, d, d, v);
    p += d * d + d;
    const float scale = 1.0f / sqrtf((float)hd);
    for (size_t h = 0; h < H; h++) {
        for (size_t i = 0; i < S; i++)
            for (size_t j = 0; j < S; j++) {
                float sum = 0.0f;
                for (size_t t = 0; t < hd; t++) sum += q[i * d + h * hd + t] * k[j * d + h * hd + t];
                float sv = sum * scale;
                if (mask && mask[i * S + j] < 0.5f) sv = -1e9f;
                sc[i * S + j] = sv;
            }
        vxo_tf_softmax_rows(sc, S, S, pr);
        for (size_t i = 0; i < S; i++)
            for (size_t t = 0; t < hd; t++) {
                float sum = 0.0f;
                for (size_t j = 0; j < S; j++) sum += pr[i * S + j] * v[j * d + h * hd + t];
                merged[i * d + h * hd + t] = sum;
            }
    }
    vxo_tf_linear(merged, S, p, p + d * d, d, d, out);
}

/* TransformerModel::forward (src/transformer.rs:773-782) with pre-norm
 * layers (TransformerLayer::forward, 647-657) */
void vxo_tf_forward(const vxo_tf_config *c, const float *params, const int64_t *tokens, size_t S, const float *mask,
                    float *logits) {
    const size_t d = c->d_model, f = c->d_ff, V = c->vocab, H = c->n_heads;
    float *pe = malloc(sizeof(float) * c->max_seq * d);
    float *x = malloc(sizeof(float) * S * d), *n1 = malloc(sizeof(float) * S * d), *a = malloc(sizeof(float) * S * d);
    float *hid = malloc(sizeof(float) * S * f), *act = malloc(sizeof(float) * S * f);
    float *scratch = malloc(sizeof(float) * (4 * S * d + 2 * S * S));
    vxo_tf_pos_encoding(c->max_seq, d, pe);
    for (size_t i = 0; i < S; i++)
        for (size_t j = 0; j < d; j++) x[i * d + j] = params[(size_t)tokens[i] * d + j] + pe[i * d + j];
    const float *p = params + V * d;
    for (size_t l = 0; l < c->n_layers; l++) {
        const float *attn = p, *l1 = p + 4 * (d * d + d), *l2 = l1 + f * d + f, *nm1 = l2 + d * f + d, *nm2 = nm1 + 2 * d;
        vxo_tf_layernorm(x, S, d, nm1, nm1 + d, 1e-5f, n1);
        tf_mha(attn, n1, S, d, H, mask, a, scratch);
        for (size_t i = 0; i < S * d; i++) x[i] = x[i] + a[i];
        vxo_tf_layernorm(x, S, d, nm2, nm2 + d, 1e-5f, n1);
        vxo_tf_linear(n1, S, l1, l1 + f * d, d, f, hid);
        vxo_tf_gelu(hid, S * f, act);
        vxo_tf_linear(act, S, l2, l2 + d * f, f, d, a);
        for (size_t i = 0; i < S * d; i++) x[i] = x[i] + a[i];
        p += 4 * (d * d + d) + (f * d + f) + (d * f + d) + 4 * d;
    }
    vxo_tf_layernorm(x, S, d, p, p + d, 1e-5f, n1);
    p += 2 * d;
    vxo_tf_linear(n1, S, p, p + V * d, d, V, logits);
    free(pe);
    free(x);
    free(n1);
    free(a);
    free(hid);
    free(act);
    free(scratch);
}
