// Internal interface of the K2 prefill GEMM (shared with the decoder).
#pragma once

#include "vxb_internal.h"

namespace vxb {

// bytes of the bf16 weight terms for an [N, K] matrix (either format)
size_t gemm_scratch_bytes(int N, int K);
// scratch of at least `bytes` owned by the context (grown with a device sync)
int gemm_ws_reserve(vxb_ctx *ctx, size_t bytes, void **out);
// Y[M, N] = X[M, K] deq(W)^T (+ resid f32 [M, N]); d_scratch holds
// gemm_scratch_bytes(N, K)
int gemm_q_launch(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x, int M, int y_dtype,
                  void *d_y, const float *d_resid, void *d_scratch, cudaStream_t st);

}  // namespace vxb
