// Pieces shared by the K1 kernels (gemv.cu: group-CTA and per-warp stream
// kernels; gemv_tc.cu: the tcgen05 kernel): stage geometry of the tiled
// layout, mbarrier / bulk-copy helpers with bounded waits, the exact code
// decoders (Q4_0 / Q8_0 to f16 or bf16 integers), scale decoding and the
// driver entry point for tensor maps. Everything has internal linkage: each
// translation unit gets its own copy.
#pragma once

#include <cstdint>
#include <mutex>

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tc_common.h"
#include "tiled_layout.h"
#include "vxb_internal.h"

namespace {

using vxb::f32_to_bf16_bits;
using vxb::ref_f16_to_f32;

constexpr int CWARPS = 8;                   // consumer warps (one 16-row tile each)
constexpr int THREADS = (CWARPS + 1) * 32;  // + one producer warp
constexpr int ROWS_PER_CTA = CWARPS * 16;
constexpr int STAGES = 3;
constexpr int CS = 4;  // chunks (units of a tile) per stage
// batches above 8: stages of 2 chunks in a 6-deep ring (the same shared
// memory, twice the look-ahead), each stage's activations as 2-D TMA boxes
// of 64 columns x B rows with 128-byte swizzle
constexpr int BCS = 2;
constexpr int BSTAGES = 6;
constexpr int XBOX_K = 64;              // columns per activation box (128 bytes)
constexpr int XBOX_BYTES = 32 * 128;    // one box, rows padded to 32 (a 1024-byte multiple)
constexpr int kMaxClusterSplits = 8;  // portable cluster size

template <int FMT>
struct Geo {
  static constexpr int CH = FMT == 0 ? 64 : 32;     // k per chunk
  static constexpr int BPC = CH / 32;               // 32-element blocks per chunk
  static constexpr int SCT = 8 * BPC * 4;           // scale bytes of one (tile, chunk) unit
  static constexpr int UNIT = 512 + SCT;            // bytes of one (tile, chunk) unit
  static constexpr int STAGE = CWARPS * CS * UNIT;  // a 128-row group's CS chunks
  // batch path: weights of one stage (1024-byte aligned) + its x boxes
  static constexpr int BW = CWARPS * BCS * UNIT;
  static constexpr int BWP = (BW + 1023) / 1024 * 1024;
  static constexpr int NXB = BCS * CH / XBOX_K;  // x boxes per stage (Q4_0 2, Q8_0 1)
  static constexpr int BSTG = BWP + NXB * XBOX_BYTES;
};
static_assert(Geo<0>::UNIT == 512 + 64 && Geo<1>::UNIT == 512 + 32, "unit size");

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// raise the transaction count without arriving
__device__ __forceinline__ void mbar_expect_tx_only(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait for the phase of the given parity (the shared helper of every
// kernel's stage rings): false after vxb::tc::kWaitBudget cycles.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  return vxb::tc::mbar_wait(bar, parity);
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t m, uint32_t o) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(m), "r"(o));
  return d;
}

__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Q4_0 tiled word -> A fragment {a0a1, a2a3, a4a5, a6a7}. Rows g (a0a1, a4a5)
// come out as the exact codes q, rows g+8 (a2a3, a6a7) as 16q.
__device__ __forceinline__ void decode_q4(uint32_t w, uint32_t A[4]) {
  const uint32_t M = 0x64006400u;       // f16 1024.0 x2
  const uint32_t SUB_LO = 0x64086408u;  // 1024 + 8
  const uint32_t SUB_HI = 0x64806480u;  // 1024 + 16 * 8
  const uint32_t w8 = w >> 8;
  A[0] = hsub2(lop_and_or(w, 0x000F000Fu, M), SUB_LO);
  A[1] = hsub2(lop_and_or(w, 0x00F000F0u, M), SUB_HI);
  A[2] = hsub2(lop_and_or(w8, 0x000F000Fu, M), SUB_LO);
  A[3] = hsub2(lop_and_or(w8, 0x00F000F0u, M), SUB_HI);
}

// Q8_0 tiled words (bytes q+128) -> A fragment of exact codes: f16 0x64uu is
// 1024 + u, minus 1152.
__device__ __forceinline__ void decode_q8(uint32_t w0, uint32_t w1, uint32_t A[4]) {
  const uint32_t M = 0x64646464u;
  const uint32_t SUB = 0x64806480u;  // 1024 + 128
  A[0] = hsub2(__byte_perm(w0, M, 0x4140), SUB);
  A[1] = hsub2(__byte_perm(w0, M, 0x4342), SUB);
  A[2] = hsub2(__byte_perm(w1, M, 0x4140), SUB);
  A[3] = hsub2(__byte_perm(w1, M, 0x4342), SUB);
}

__device__ __forceinline__ uint32_t bsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// bf16 operands (batches above 8, activations staged unchanged). Q4_0: nibble
// n at bits 0-3 / 16-19 of (w >> 4i) gives bf16 0x4300|n = 128+n, minus 136:
// the exact codes of every row.
__device__ __forceinline__ void decode_q4_bf16(uint32_t w, uint32_t A[4]) {
  const uint32_t M = 0x43004300u;    // bf16 128.0 x2
  const uint32_t SUB = 0x43084308u;  // bf16 136.0 x2
  A[0] = bsub2(lop_and_or(w, 0x000F000Fu, M), SUB);
  A[1] = bsub2(lop_and_or(w >> 4, 0x000F000Fu, M), SUB);
  A[2] = bsub2(lop_and_or(w >> 8, 0x000F000Fu, M), SUB);
  A[3] = bsub2(lop_and_or(w >> 12, 0x000F000Fu, M), SUB);
}

// Q8_0 bytes u = q+128 -> f32 2^23+u by PRMT, minus 2^23+128, packed to bf16
// (exact: |q| <= 128)
__device__ __forceinline__ void q8_word_bf16(uint32_t w, uint32_t &lo, uint32_t &hi) {
  const float Bm = 8388736.0f;  // 2^23 + 128
  const float c0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440)) - Bm;
  const float c1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441)) - Bm;
  const float c2 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442)) - Bm;
  const float c3 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443)) - Bm;
  lo = pack_bf16x2(c0, c1);
  hi = pack_bf16x2(c2, c3);
}

__device__ __forceinline__ void decode_q8_bf16(uint32_t w0, uint32_t w1, uint32_t A[4]) {
  q8_word_bf16(w0, A[0], A[1]);
  q8_word_bf16(w1, A[2], A[3]);
}

__device__ __forceinline__ void mma_bf16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16_z(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

__device__ __forceinline__ void mma_f16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// the same with a zero accumulator input
__device__ __forceinline__ void mma_f16_z(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

__device__ __forceinline__ float2 decode_scales(uint32_t s, bool subnormal) {
  if (!subnormal) {
    __half2 h = *reinterpret_cast<__half2 *>(&s);
    return __half22float2(h);
  }
  return make_float2(ref_f16_to_f32(s & 0xFFFFu), ref_f16_to_f32(s >> 16));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// v * 2^e for |e| <= 252: two exact power-of-two factors (exact unless the
// result leaves the f32 range)
__device__ __forceinline__ float mul_pow2(float v, int e) {
  const int e1 = e / 2, e2 = e - e1;
  return v * __int_as_float((127 + e1) << 23) * __int_as_float((127 + e2) << 23);
}

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(src_bytes));
}

// all threads of every CTA of the cluster (release / acquire)
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
  static std::mutex mu;
  static EncodeTiledFn fn = nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p) {
      cudaGetLastError();
      return nullptr;
    }
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Tensor map of the activations x [B, K] bf16 for the batch path: boxes of
// 64 columns x B rows, 128-byte swizzle, columns past K read as zero.
inline int x_tensor_map(vxb_ctx *ctx, const uint16_t *x, int B, int K, CUtensorMap *map) {
  const EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return vxb::set_error(ctx, VXB_ECUDA, "vxb_gemv_q: cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)B};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)XBOX_K, (cuuint32_t)B};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return vxb::set_error(ctx, VXB_EINVAL, "vxb_gemv_q: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VXB_OK;
}

}  // namespace
