/*
 * vxo.h -- CPU oracle for the quantized-inference hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library restates, in plain C, the CPU
 * arithmetic of the reference (MangoByteLabs/vortex, Rust) for the path that
 * the vortex_b200 CUDA kernels replace. It is used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline / reference arm as
 * the reference to compare against and the CPU baseline -- never by the
 * product path.
 *
 * Every function cites the reference file:line it follows. Loop orders are
 * kept as in the reference so f64 results are reproducible.
 */
#ifndef VXO_H
#define VXO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* quantize.rs QuantFormat subset used on the path */
enum { VXO_INT8 = 0, VXO_INT4 = 1, VXO_INT2 = 2 };
/* gguf_loader.rs GGMLQuantType values (src/gguf_loader.rs:61-75) */
enum { VXO_GGML_F32 = 0, VXO_GGML_F16 = 1, VXO_GGML_Q4_0 = 2, VXO_GGML_Q4_1 = 3, VXO_GGML_Q8_0 = 8 };

/* ---- f16 / bf16 bit conversions (src/tensor_engine.rs:42-103) ---- */
uint16_t vxo_f32_to_f16(float x);
float vxo_f16_to_f32(uint16_t h);
uint16_t vxo_f32_to_bf16(float x);
float vxo_bf16_to_f32(uint16_t b);

/* ---- calibration (src/quantize.rs:585-600) ---- */
double vxo_calibrate_minmax(const double *data, size_t n);
double vxo_calibrate_minmax_range(const double *data, size_t n, double qmin, double qmax);

/* ---- packing (src/quantize.rs:664-722) ---- */
void vxo_pack_int4(const int8_t *values, size_t n, uint8_t *out);      /* out: (n+1)/2 bytes */
void vxo_unpack_int4(const uint8_t *packed, size_t nbytes, int8_t *out); /* out: 2*nbytes */
void vxo_pack_int2(const int8_t *values, size_t n, uint8_t *out);      /* out: (n+3)/4 bytes */
void vxo_unpack_int2(const uint8_t *packed, size_t nbytes, int8_t *out); /* out: 4*nbytes */

/* ---- QuantTensor::quantize / dequantize (src/quantize.rs:81-235, 312-444) ----
 * group_size == 0 means PerTensor. Returns the number of packed bytes written.
 * scales / zps receive one entry per group (one entry for PerTensor). */
size_t vxo_quantize(const double *data, size_t n, int fmt, size_t group_size,
                    uint8_t *packed, double *scales, int64_t *zps);
size_t vxo_num_groups(size_t n, size_t group_size);
void vxo_dequantize(const uint8_t *packed, size_t nbytes, size_t numel, int fmt,
                    size_t group_size, const double *scales, const int64_t *zps,
                    double *out);
/* QuantTensor::get_scale: mean of group scales (src/quantize.rs:534-545) */
double vxo_get_scale(const double *scales, size_t n_scales, int per_group);
/* QuantTensor::matmul_int8 / matmul_int4 (src/quantize.rs:473-515): A [m,k], B [k,n] */
void vxo_matmul_int(const uint8_t *a, const uint8_t *b, int fmt, size_t m, size_t k, size_t n,
                    double a_scale, double b_scale, int64_t a_zp, int64_t b_zp, double *out);
/* matmul_f64 (src/quantize.rs:890-902) */
void vxo_matmul_f64(const double *a, const double *b, size_t m, size_t k, size_t n, double *out);

/* ---- GGUF block dequantization (src/gguf_loader.rs:413-531) ---- */
void vxo_dequantize_q4_0(const uint8_t *data, size_t n, float *out);
void vxo_dequantize_q4_1(const uint8_t *data, size_t n, float *out);
void vxo_dequantize_q8_0(const uint8_t *data, size_t n, float *out);
size_t vxo_dequantize_f16(const uint8_t *data, size_t nbytes, size_t n, float *out);
size_t vxo_copy_f32(const uint8_t *data, size_t nbytes, size_t n, float *out);
size_t vxo_ggml_data_size(int ggml_type, size_t n_elements); /* GGUFTensorInfo::data_size */

/* ---- composed Q8_0 / Q4_0 block quantizer ----
 * codes: quantize.rs PerGroup rules (group 32 over the flat buffer);
 * storage: gguf_loader.rs block layout; scale: f64 -> f32 -> f32_to_f16. */
void vxo_quantize_q8_0(const double *w, size_t n, uint8_t *blocks);
void vxo_quantize_q4_0(const double *w, size_t n, uint8_t *blocks);

/* y[b*N + r] = sum_k deq(W)[r*K + k] * x[b*K + k], f64, W given as GGUF blocks */
void vxo_gemv_blocks(int ggml_type, const uint8_t *blocks, size_t N, size_t K,
                     const double *x, size_t B, double *y);

/* ---- attention (src/flash_attention.rs:22-219, 519-564) ---- */
int vxo_flash_auto_tile(size_t seq_len, size_t head_dim);
void vxo_flash_attention_forward(const double *q, const double *k, const double *v,
                                 size_t n, size_t d, size_t br, size_t bc, int causal,
                                 double *out, double *lse, double *row_max);
void vxo_flash_attention_backward(const double *q, const double *k, const double *v, const double *out,
                                  const double *grad_out, const double *lse, size_t n, size_t d, size_t br,
                                  size_t bc, int causal, double *grad_q, double *grad_k, double *grad_v);
void vxo_standard_attention(const double *q, const double *k, const double *v,
                            size_t n, size_t d, int causal, double *out);
void vxo_multi_head_flash_attention(const double *q, const double *k, const double *v,
                                    size_t n, size_t num_heads, size_t head_dim, int causal,
                                    double *out);
/* Exact softmax attention for selected query rows of one head, [n,d] inputs,
 * scale 1/sqrt(d) as flash_attention_forward; also returns lse per row. */
void vxo_attention_rows(const double *q, const double *k, const double *v, size_t n, size_t d,
                        int causal, const int64_t *rows, size_t nrows, double *out, double *lse);

/* ---- paged decode attention (src/kv_cache.rs:95-112) ---- */
void vxo_paged_attention(const double *query, const double *keys, const double *values,
                         size_t ctx, size_t head_dim, double *out);

/* ---- Llama-style block math (stdlib/ai/transformer.vx:413-603) ---- */
void vxo_rmsnorm_bias(const double *x, const double *w, const double *b, size_t n, double eps,
                      double *out);
void vxo_rope_embed(const double *x, size_t n, int64_t pos, int64_t dim, double *out);
void vxo_rope_builtin(const double *x, size_t n, const double *freqs, size_t n_freqs, double *out);
void vxo_vec_add(const double *a, const double *b, size_t n, double *out);
double vxo_silu(double x);
void vxo_matvec(const double *w, const double *v, size_t out_dim, size_t in_dim, double *out);

/* ---- f32 GPT-style model (src/transformer.rs:15-841), oracle/vxo_tf.c ---- */
typedef struct {
    size_t vocab, d_model, n_heads, n_layers, d_ff, max_seq;
} vxo_tf_config;
size_t vxo_tf_param_count(const vxo_tf_config *c);
void vxo_tf_init(const vxo_tf_config *c, uint64_t seed, float *params);
void vxo_tf_pos_encoding(size_t max_len, size_t d, float *out);
void vxo_tf_linear(const float *x, size_t m, const float *w, const float *b, size_t in, size_t out, float *y);
void vxo_tf_layernorm(const float *x, size_t rows, size_t d, const float *g, const float *b, float eps, float *y);
void vxo_tf_gelu(const float *x, size_t n, float *y);
void vxo_tf_softmax_rows(const float *x, size_t rows, size_t cols, float *y);
void vxo_tf_forward(const vxo_tf_config *c, const float *params, const int64_t *tokens, size_t S, const float *mask,
                    float *logits);

/* ---- sampling (stdlib/ai/transformer.vx:36-80, 1163-1260), oracle/vxo_sample.c ---- */
double vxo_vx_exp(double x);
int64_t vxo_argmax(const double *logits, size_t n);
double vxo_lcg_uniform(int64_t seed);
int64_t vxo_sample_top_p(const double *logits, size_t n, double temperature, double top_p, int64_t seed);

/* ---- int dot primitives (src/bytecarry.rs:491-513) ---- */
int32_t vxo_int8_dot(const int8_t *a, const int8_t *b, size_t n);
int32_t vxo_int4_dot(const uint8_t *a, const uint8_t *b, size_t nbytes);

#ifdef __cplusplus
}
#endif
#endif
