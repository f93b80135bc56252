// Internal interface of the decoder's small kernels.
#pragma once

#include "kv_cache.h"

namespace vxb {

int rmsnorm_launch(vxb_ctx *ctx, const float *x, const float *w, const float *b, int rows, int n, float eps,
                   uint16_t *out, cudaStream_t st);
// RoPE of rows of f32 (q | k | v) projections fused with the KV-cache
// append of layer `layer` at places[row] (kv null: no cache write): q to
// q_out, k and v also to k_lin / v_lin when non-null (bf16 [rows, kvdim]).
// q/k rotation pairs are numbered from q_pair0 / k_pair0 (tensor-parallel
// slices of the heads).
int rope_kv_launch(vxb_ctx *ctx, vxb_kv *kv, int layer, const float *qkv, int rows, int qdim, int kvdim, int hd,
                   const KVPlace *places, const double *rope_div, uint16_t *q_out, uint16_t *k_lin, uint16_t *v_lin,
                   int q_pair0, int k_pair0, cudaStream_t st);
int swiglu_launch(vxb_ctx *ctx, const float *gu, int rows, int ffn, uint16_t *act, cudaStream_t st);
int embed_launch(vxb_ctx *ctx, const uint16_t *emb, const int32_t *tokens, int rows, int dim, int vocab, float *x,
                 cudaStream_t st);
int argmax_launch(vxb_ctx *ctx, const float *logits, int rows, int vocab, int32_t *out, cudaStream_t st);
int normal_fill(vxb_ctx *ctx, float *out, size_t n, uint64_t seed, size_t offset, float sigma, cudaStream_t st);
// block [rows, cols] at (row0, col0) of the matrix normal_fill makes with leading dimension ld
int normal_fill_block(vxb_ctx *ctx, float *out, int rows, int cols, size_t row0, size_t col0, size_t ld, uint64_t seed,
                      float sigma, cudaStream_t st);
// distributed greedy argmax: per-row key of the shard's first maximum (global
// index = offset + local), and the token of a (max-reduced) key
int argmax_key_launch(vxb_ctx *ctx, const float *logits, int rows, int vocab, int offset, unsigned long long *keys,
                      cudaStream_t st);
int key_to_token_launch(vxb_ctx *ctx, const unsigned long long *keys, int rows, int32_t *out, cudaStream_t st);
int unshard_launch(vxb_ctx *ctx, const float *in, int tp, int rows, int shard, float *out, cudaStream_t st);

}  // namespace vxb
