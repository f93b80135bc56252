// Internal interface of the decoder's small kernels.
#pragma once

#include "kv_cache.h"

namespace vxb {

int rmsnorm_launch(vxb_ctx *ctx, const float *x, const float *w, const float *b, int rows, int n, float eps,
                   uint16_t *out, cudaStream_t st);
int rope_launch(vxb_ctx *ctx, const float *qkv, int rows, int dim, int kvdim, const KVPlace *places,
                const double *rope_div, uint16_t *q_out, uint16_t *k_out, uint16_t *v_out, cudaStream_t st);
int swiglu_launch(vxb_ctx *ctx, const float *gu, int rows, int ffn, uint16_t *act, cudaStream_t st);
int embed_launch(vxb_ctx *ctx, const uint16_t *emb, const int32_t *tokens, int rows, int dim, int vocab, float *x,
                 cudaStream_t st);
int argmax_launch(vxb_ctx *ctx, const float *logits, int rows, int vocab, int32_t *out, cudaStream_t st);
int normal_fill(vxb_ctx *ctx, float *out, size_t n, uint64_t seed, size_t offset, float sigma, cudaStream_t st);

}  // namespace vxb
