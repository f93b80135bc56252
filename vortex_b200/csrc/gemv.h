// Internal interface of the K1 GEMV (shared with the decoder).
#pragma once

#include "vxb_internal.h"

namespace vxb {

struct GemvPlan {
  int S;        // k-splits (CTAs per row group)
  bool pdl;      // launch with programmatic stream serialization
  bool cluster;  // the splits of a row group form a cluster (S <= 8)
};

GemvPlan gemv_plan(const vxb_ctx *ctx, int fmt, int N, int K, int batch);
size_t gemv_smem_bytes(int fmt, int N, int K, int batch, int S);

// y = W x (+ resid). d_resid (optional) is f32 [batch, N] added in the epilogue.
int gemv_launch(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x, int batch,
                int y_dtype, void *d_y, const float *d_resid, void *stream, const GemvPlan *plan_override);

// Batches 9..32 on the tcgen05 kernel (gemv_tc.cu): by default Q4_0 batches
// 17-32 and Q8_0 batches 9-32 with up to 16384 rows, batches 28-32 with more
// rows, and Q8_0 with 28000 rows or more (VXB_GEMV_TCGEN05=1: every
// batch 9-32, =0: none). d_err is the device error word.
bool gemv_tc_eligible(int fmt, int N, int batch);
int gemv_tc_splits(const vxb_ctx *ctx, int fmt, int N, int K, int batch);
int gemv_tc(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x, int batch, int y_dtype,
            void *d_y, const float *d_resid, int *d_err, cudaStream_t st, bool pdl);

// Error word of vxb_gemv_q_static's fixed array on a device: null while the
// array has not been resolved there; the _resolve form resolves it.
int *static_error_word(int device);
int static_error_word_resolve(vxb_ctx *ctx, int **out);

}  // namespace vxb
