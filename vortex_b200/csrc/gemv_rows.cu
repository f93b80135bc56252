// GEMV over GGUF tensors stored as they are in the file (row-major rows of
// blocks), for every GGUF type the reference dequantizes: F32, F16, Q4_0,
// Q4_1, Q8_0 (src/gguf_loader.rs:413-531):
//
//   y[b, n] = sum_k deq(W)[n, k] * x[b, k]
//
// This is the path for tensors the tiled kernels do not take (Q4_1, F16,
// F32 - e.g. a GGUF whose projections are Q4_1); Q4_0 / Q8_0 are accepted too
// but run faster tiled (vxb_tile_weights + vxb_gemv_q). Each warp owns one
// row; lane j handles blocks j, j + 32, ... of the row, so a warp reads 32
// consecutive blocks (20 to 128 bytes each) per step, coalesced. The
// activations of a k-tile are staged once per CTA in shared memory as f32,
// up to 8 batch rows per pass (larger batches take several passes over the
// weights). Every weight is the reference's f32 dequantized value (the same
// decode as vxb_dequantize_blocks); products accumulate in f32, the lanes'
// sums add in a fixed butterfly order.
#include "vxb_internal.h"

using namespace vxb;

namespace {

constexpr int GR_WARPS = 8;       // rows per CTA
constexpr int GR_KT = 1024;       // k per shared-memory tile
constexpr int GR_KP = GR_KT + GR_KT / 32;  // padded: element k at k + k / 32 (lanes read conflict-free)
constexpr int GR_BMAX = 8;        // batch rows per pass

struct RowsArgs {
  const uint8_t *w;
  const uint16_t *x;
  void *y;
  int type, N, K, B, b0, nb, y_dtype;
  size_t row_bytes;
};

__device__ __forceinline__ uint32_t u16_at(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// the 32 values of block `blk` of a row (elements blk*32 .. blk*32+31; past K
// the caller's x is zero, so any finite value is harmless - F16/F32 rows stop
// at K and read nothing beyond it)
__device__ __forceinline__ void decode_block(const RowsArgs &a, const uint8_t *row, int blk, float (&w)[32]) {
  if (a.type == VXB_Q4_0 || a.type == VXB_Q4_1) {
    const bool q41 = a.type == VXB_Q4_1;
    const uint8_t *b = row + (size_t)blk * (q41 ? 20 : 18);
    const float d = ref_f16_to_f32(u16_at(b));
    const float m = q41 ? ref_f16_to_f32(u16_at(b + 2)) : 0.f;
    const uint8_t *q = b + (q41 ? 4 : 2);
#pragma unroll
    for (int j = 0; j < 16; j++) {
      const int byte = q[j];
      if (q41) {
        w[2 * j] = __fadd_rn(__fmul_rn((float)(byte & 0xF), d), m);
        w[2 * j + 1] = __fadd_rn(__fmul_rn((float)(byte >> 4), d), m);
      } else {
        w[2 * j] = __fmul_rn((float)((byte & 0xF) - 8), d);
        w[2 * j + 1] = __fmul_rn((float)((byte >> 4) - 8), d);
      }
    }
  } else if (a.type == VXB_Q8_0) {
    const uint8_t *b = row + (size_t)blk * 34;
    const float d = ref_f16_to_f32(u16_at(b));
#pragma unroll
    for (int j = 0; j < 32; j++) w[j] = __fmul_rn((float)(int8_t)b[2 + j], d);
  } else if (a.type == VXB_GGML_F16) {
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const int k = blk * 32 + j;
      w[j] = k < a.K ? ref_f16_to_f32(u16_at(row + 2 * (size_t)k)) : 0.f;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const int k = blk * 32 + j;
      w[j] = k < a.K ? __ldg(reinterpret_cast<const float *>(row) + k) : 0.f;
    }
  }
}

__global__ void __launch_bounds__(GR_WARPS * 32) gemv_rows_kernel(const RowsArgs a) {
  __shared__ float xs[GR_BMAX][GR_KP];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * GR_WARPS + warp;
  const uint8_t *row = a.w + (size_t)(r < a.N ? r : 0) * a.row_bytes;
  float acc[GR_BMAX];
#pragma unroll
  for (int j = 0; j < GR_BMAX; j++) acc[j] = 0.f;
  for (int k0 = 0; k0 < a.K; k0 += GR_KT) {
    const int kt = min(GR_KT, a.K - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < a.nb * GR_KT; i += blockDim.x) {
      const int b = i / GR_KT, k = i % GR_KT;
      xs[b][k + k / 32] = k < kt ? bf16_bits_to_f32(__ldg(a.x + (size_t)(a.b0 + b) * a.K + k0 + k)) : 0.f;
    }
    __syncthreads();
    if (r < a.N) {
      for (int blk = k0 / 32 + lane; blk * 32 < k0 + kt; blk += 32) {
        float w[32];
        decode_block(a, row, blk, w);
        const int kk = blk * 32 - k0;
#pragma unroll
        for (int j = 0; j < GR_BMAX; j++) {
          if (j < a.nb) {
            float s = 0.f;
#pragma unroll
            for (int e = 0; e < 32; e++) s = __fmaf_rn(w[e], xs[j][kk + kk / 32 + e], s);
            acc[j] += s;
          }
        }
      }
    }
  }
  if (r >= a.N) return;
#pragma unroll
  for (int j = 0; j < GR_BMAX; j++) {
    if (j >= a.nb) break;
    const float v = warp_sum(acc[j]);
    if (lane == 0) {
      const size_t o = (size_t)(a.b0 + j) * a.N + r;
      if (a.y_dtype == VXB_BF16)
        reinterpret_cast<uint16_t *>(a.y)[o] = f32_to_bf16_bits(v);
      else
        reinterpret_cast<float *>(a.y)[o] = v;
    }
  }
}

}  // namespace

VXB_API int vxb_gemv_blocks(vxb_ctx *ctx, int type, const void *d_rows, int N, int K, const uint16_t *d_x, int batch,
                            int y_dtype, void *d_y, void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_gemv_blocks: null context");
  const bool blocked = type == VXB_Q4_0 || type == VXB_Q4_1 || type == VXB_Q8_0;
  if (!blocked && type != VXB_GGML_F16 && type != VXB_GGML_F32)
    return set_error(ctx, VXB_EINVAL, "vxb_gemv_blocks: unknown GGUF type %d", type);
  if (N <= 0 || K <= 0 || (blocked && K % 32) || batch < 1)
    return set_error(ctx, VXB_EINVAL, "vxb_gemv_blocks: bad shape N=%d K=%d batch=%d", N, K, batch);
  if (y_dtype != VXB_F32 && y_dtype != VXB_BF16) return set_error(ctx, VXB_EINVAL, "vxb_gemv_blocks: y_dtype");
  if (!d_rows || !d_x || !d_y) return set_error(ctx, VXB_EINVAL, "vxb_gemv_blocks: null pointer");
  if (type == VXB_GGML_F32 && (uintptr_t)d_rows % 4)
    return set_error(ctx, VXB_EINVAL, "vxb_gemv_blocks: F32 rows must be 4-byte aligned");
  if (int rc = use_device(ctx)) return rc;
  RowsArgs a;
  a.w = (const uint8_t *)d_rows;
  a.x = d_x;
  a.y = d_y;
  a.type = type;
  a.N = N;
  a.K = K;
  a.B = batch;
  a.y_dtype = y_dtype;
  a.row_bytes = vxb_block_bytes(type, (size_t)K);
  if (type == VXB_GGML_F32 && a.row_bytes % 4) return set_error(ctx, VXB_EINVAL, "vxb_gemv_blocks: F32 row size");
  cudaStream_t st = (cudaStream_t)stream;
  for (int b0 = 0; b0 < batch; b0 += GR_BMAX) {
    a.b0 = b0;
    a.nb = batch - b0 < GR_BMAX ? batch - b0 : GR_BMAX;
    gemv_rows_kernel<<<(N + GR_WARPS - 1) / GR_WARPS, GR_WARPS * 32, 0, st>>>(a);
    if (int rc = launch_check(ctx, "gemv_rows_kernel")) return rc;
  }
  return VXB_OK;
}
