// Internal declarations shared by the vortex_b200 CUDA sources.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/vxb.h"

#define VXB_API extern "C" __attribute__((visibility("default")))

struct vxb_ctx {
  int device = 0;
  int num_sms = 0;
  size_t smem_optin = 0;
  std::string err;
  // split-K partials and reduction counters, grown on demand (see ws_reserve)
  void *ws = nullptr;
  size_t ws_bytes = 0;
  unsigned *counters = nullptr;  // zero-initialised; kernels restore zero after use
  size_t n_counters = 0;
  // device error word: kernels whose bounded waits time out set it to nonzero
  int *d_err = nullptr;
  // bf16 hi/lo weight copies of the prefill GEMM (vxb_gemm_q), grown on demand
  void *gemm_ws = nullptr;
  size_t gemm_ws_bytes = 0;
};

namespace vxb {

// Record an error message on ctx (or globally when ctx is null) and return code.
int set_error(vxb_ctx *ctx, int code, const char *fmt, ...) __attribute__((format(printf, 3, 4)));

// Translate a CUDA error into VXB_ECUDA with a message naming the call site.
int cuda_fail(vxb_ctx *ctx, cudaError_t e, const char *what);

#define VXB_CUDA_TRY(ctx, call)                                   \
  do {                                                            \
    cudaError_t _e = (call);                                      \
    if (_e != cudaSuccess) return vxb::cuda_fail((ctx), _e, #call); \
  } while (0)

// Make the context's device current for this host thread.
int use_device(vxb_ctx *ctx);

// Ensure the workspace holds `bytes` and `counters` reduction counters.
// Allocation happens only when growing, so calls that fit the current size
// (for example inside CUDA graph capture) allocate nothing.
int ws_reserve(vxb_ctx *ctx, size_t bytes, size_t counters);

inline size_t round_up(size_t x, size_t m) { return (x + m - 1) / m * m; }

// Tiled weight layout (blocks.cu): write the header of a [N, K] layout, and
// tile `nrows` rows of GGUF blocks into rows [row0, row0 + nrows) of a layout
// whose full height is N_total (row0 a multiple of 16).
int tile_header(vxb_ctx *ctx, int fmt, int N, int K, void *d_tiled, cudaStream_t st);
int tile_part(vxb_ctx *ctx, int fmt, const uint8_t *d_blocks, int nrows, int K, int row0, int N_total, void *d_tiled,
              cudaStream_t st);

// Launch-error check after a kernel launch.
inline int launch_check(vxb_ctx *ctx, const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  return VXB_OK;
}

}  // namespace vxb

// ------------------------------------------------------------------------
// Device helpers
// ------------------------------------------------------------------------
#ifdef __CUDACC__
namespace vxb {

// tensor_engine::f16_to_f32 (src/tensor_engine.rs:66-92) for one f16 bit
// pattern, including its subnormal decoding (exponent 127-15-e, i.e. half the
// IEEE value: frac * 2^-25).
__device__ __forceinline__ float ref_f16_to_f32(uint32_t h) {
  uint32_t sign = (h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t frac = h & 0x3FFu;
  if (exp == 0) {
    float m = (float)frac * 2.98023223876953125e-08f;  // 2^-25
    return __uint_as_float(__float_as_uint(m) | sign);
  }
  if (exp == 31) return __uint_as_float(sign | 0x7F800000u | (frac << 13));
  return __uint_as_float(sign | ((exp + 112u) << 23) | (frac << 13));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// tensor_engine::f32_to_bf16 (src/tensor_engine.rs:94-99): RNE via bias.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
  uint32_t bits = __float_as_uint(x);
  uint32_t bias = 0x7FFFu + ((bits >> 16) & 1u);
  return (uint16_t)((bits + bias) >> 16);
}

// tensor_engine::f32_to_f16 (src/tensor_engine.rs:42-64): truncating.
__device__ __forceinline__ uint16_t f32_to_f16_trunc(float x) {
  uint32_t bits = __float_as_uint(x);
  uint32_t sign = (bits >> 16) & 0x8000u;
  int exp = (int)((bits >> 23) & 0xFFu);
  uint32_t frac = bits & 0x7FFFFFu;
  if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (frac != 0 ? 0x200u : 0u));
  int ne = exp - 127 + 15;
  if (ne >= 31) return (uint16_t)(sign | 0x7C00u);
  if (ne <= 0) {
    if (ne < -10) return (uint16_t)sign;
    uint32_t f = (frac | 0x800000u) >> (uint32_t)(1 - ne);
    return (uint16_t)(sign | (f >> 13));
  }
  return (uint16_t)(sign | ((uint32_t)ne << 10) | (frac >> 13));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace vxb
#endif
