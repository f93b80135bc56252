// K1: decode dequant-GEMV / skinny GEMM over tiled Q4_0 / Q8_0 weights.
//
//   y[b, n] = sum_k deq(W)[n, k] * x[b, k]     (b < batch <= 32)
//
// Replaces weight_only_matmul (src/quantize.rs:845-852, = dequantize then
// matmul_f64 890-902) and the matmul of Linear::forward
// (src/transformer.rs:332-352) at decode batch sizes.
//
// Design (HBM-bound streaming):
//  * A CTA owns one 128-row group (8 sixteen-row tiles, one per consumer warp)
//    and a k-range. The tiled layout stores every (row group, k-chunk) as one
//    contiguous record of codes and scales, so a producer warp moves a whole
//    stage (CS records) with a single cp.async.bulk copy into a ring of
//    shared-memory stages (one mbarrier per stage with a transaction count).
//  * Consumer warps read their tile's codes with one 16-byte LDS per lane per
//    chunk (the slice is the lane's m16n8k16 A fragments) and turn them into
//    exact f16 integers: Q4_0 nibbles by LOP3 with the f16 magic 1024 (a nibble
//    at bits 0-3 gives 1024+n, at bits 4-7 1024+16n) and one HSUB2 per two
//    codes; Q8_0 bytes (stored as q+128) by one PRMT with the magic byte and one
//    HSUB2 per two codes.
//  * The activations of the CTA's k-range are staged in shared memory as f16,
//    each batch column multiplied by a power of two 2^-e chosen from its largest
//    magnitude (max |x| * 2^-e in [2^14, 2^15)), so the bf16 -> f16 conversion is
//    exact for every element within 2^-28 of the column maximum and nothing
//    overflows; the f32 result is multiplied back by 2^e.
//  * mma.m16n8k16 (f16 x f16 -> f32) forms the per-block dot products; the
//    per-(row, block) f16 scale multiplies that f32 block partial with packed
//    f32x2 FMAs, so scales never round into the operands (Q4_0 rows decoded as
//    16q carry 1/16 in their scale, an exact factor).
//  * Split-K across CTAs with a deterministic reduction: each CTA writes its
//    f32 partial and the last CTA of a row group (counter in global memory)
//    sums the partials in split order and applies the epilogue; the counter is
//    returned to zero.
//  * The producer issues weight copies before any dependency on the kernel
//    that produces x, so under programmatic dependent launch the weight stream
//    overlaps the producer kernel's tail. Every mbarrier wait is bounded
//    (clock64); a timeout sets the context's device error word and the kernel
//    runs to completion.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>

#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gemv.h"
#include "tc_common.h"
#include "tiled_layout.h"
#include "vxb_internal.h"

using namespace vxb;
namespace cg = cooperative_groups;

namespace {

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

// Activations: batches up to 8 (XF16) stage the split's x once as f16 scaled
// per batch column by 2^-e; larger batches carry an unchanged bf16 x slice in
// every stage (no prologue, shared memory independent of K).
template <int NT>
struct XMode {
  static constexpr bool F16 = NT == 1;
};
static_assert(Geo<0>::UNIT == 512 + 64 && Geo<1>::UNIT == 512 + 32, "unit size");

struct GemvArgs {
  const uint8_t *records;
  const uint32_t *hdr;
  const uint16_t *x;
  void *y;
  const float *resid;  // optional residual added in the epilogue (f32 [B, N])
  float *ws;
  unsigned *counters;
  int *err;
  int N, K, B, NP, n_chunks, S, y_dtype, xs_stride;
  int cluster;  // 1: the S splits of a row group are one thread-block cluster
};

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

// Bounded wait for the phase of the given parity; false after ~2^31 cycles.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > (1ll << 31)) return false;
  }
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

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(CWARPS * 32) : "memory"); }

__device__ __forceinline__ void epilogue_store(const GemvArgs &a, int b, int row, float v) {
  const size_t o = (size_t)b * a.N + row;
  if (a.resid) v += __ldcg(a.resid + o);
  if (a.y_dtype == VXB_BF16)
    ((uint16_t *)a.y)[o] = f32_to_bf16_bits(v);
  else
    ((float *)a.y)[o] = v;
}

// Consumer main loop over n_iter full stages: acc[nt][0] = rows g, acc[nt][1]
// = rows g+8 of the warp's tile, batch columns (2q, 2q+1) of n-tile nt.
// Batch <= 8: stages of CS chunks, x staged once for the split as f16 (xs).
// Batch > 8: stages of BCS chunks whose activations follow the weights as
// swizzled TMA boxes (row n of a box at n * 128 bytes, 16-byte chunk c of the
// row at chunk position c ^ (n % 8)).
template <int FMT, int NT, bool SUBN>
__device__ __forceinline__ void consume_stages(const GemvArgs &a, const uint8_t *stages, uint64_t *full,
                                               uint64_t *empty, const uint16_t *xs, int n_iter, float2 (&acc)[NT][2]) {
  using G = Geo<FMT>;
  constexpr bool XF16 = XMode<NT>::F16;
  constexpr int KCS = XF16 ? CS : BCS;          // chunks per stage
  constexpr int NSTG = XF16 ? STAGES : BSTAGES;  // ring depth
  constexpr int STG = XF16 ? G::STAGE : G::BSTG;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int nt = 0; nt < NT; nt++) acc[nt][0] = acc[nt][1] = make_float2(0.f, 0.f);
  const int xlane = (lane >> 2) * a.xs_stride + (lane & 3) * 4;  // XF16
  // batch path: byte offset of the lane's 8-byte operand inside a box, for
  // the four 16-column positions C = 0, 2, 4, 6 of the 16-byte chunk index
  // ((C | (q >> 1)) ^ n) with n % 8 = lane / 4 for every n-tile
  uint32_t boff[4];
  {
    const int q = lane & 3, sw = lane >> 2;
#pragma unroll
    for (int c = 0; c < 4; c++)
      boff[c] = (uint32_t)(sw * 128 + ((((2 * c) | (q >> 1)) ^ sw) << 4) + (q & 1) * 8);
  }
  // batch rows past B are not staged: their operand is zero
  bool live[NT];
#pragma unroll
  for (int nt = 0; nt < NT; nt++) live[nt] = nt * 8 + (lane >> 2) < a.B;

  // Blocks of a stage are processed in groups of GB with independent
  // accumulators: the first k16 step of every block of the group is issued,
  // then the second, then the scale FMAs, so consecutive MMAs never depend on
  // each other and the tensor-core latency overlaps across blocks.
  constexpr int BLK = KCS * G::BPC;                          // blocks per stage
  constexpr int GB0 = NT == 1 ? 4 : (NT == 2 ? 2 : 1);
  constexpr int GB = GB0 < BLK ? GB0 : BLK;                   // blocks per group
  for (int it = 0; it < n_iter; it++) {
    const int slot = it % NSTG;
    if (!mbar_wait(&full[slot], (it / NSTG) & 1)) atomicExch(a.err, 1);
    const uint8_t *st = stages + slot * STG;
    const uint8_t *cw = st + warp * KCS * G::UNIT + lane * 16;
    const uint8_t *sw = st + warp * KCS * G::UNIT + 512 + (lane >> 2) * G::BPC * 4;
    uint4 wv[KCS];
    uint32_t sv[KCS][G::BPC];
#pragma unroll
    for (int j = 0; j < KCS; j++) {
      wv[j] = *reinterpret_cast<const uint4 *>(cw + j * G::UNIT);
      if (G::BPC == 2) {
        const uint2 t2 = *reinterpret_cast<const uint2 *>(sw + j * G::UNIT);
        sv[j][0] = t2.x;
        sv[j][G::BPC - 1] = t2.y;
      } else {
        sv[j][0] = *reinterpret_cast<const uint32_t *>(sw + j * G::UNIT);
      }
    }
    const uint16_t *xk = xs + it * CS * G::CH + xlane;  // XF16
    const uint8_t *xbox = st + G::BWP;                   // batch path
#pragma unroll
    for (int b0 = 0; b0 < BLK; b0 += GB) {
      float t[GB][NT][4];
#pragma unroll
      for (int h = 0; h < 2; h++) {
#pragma unroll
        for (int gb = 0; gb < GB; gb++) {
          const int blk = b0 + gb, j = blk / G::BPC, bb = blk % G::BPC;
          const uint32_t *wu = reinterpret_cast<const uint32_t *>(&wv[j]);
          uint32_t A[4];
          if (XF16) {
            if (FMT == 0)
              decode_q4(wu[bb * 2 + h], A);
            else
              decode_q8(wu[h * 2], wu[h * 2 + 1], A);
          } else {
            if (FMT == 0)
              decode_q4_bf16(wu[bb * 2 + h], A);
            else
              decode_q8_bf16(wu[h * 2], wu[h * 2 + 1], A);
          }
          // column of this k16 step inside the stage, its box and 16-column position
          const int kk = blk * 32 + h * 16;
#pragma unroll
          for (int nt = 0; nt < NT; nt++) {
            uint2 bx = make_uint2(0u, 0u);
            if (live[nt]) {
              if (XF16)
                bx = *reinterpret_cast<const uint2 *>(xk + (size_t)nt * 8 * a.xs_stride + kk);
              else
                bx = *reinterpret_cast<const uint2 *>(xbox + (kk / XBOX_K) * XBOX_BYTES + nt * 8 * 128 +
                                                      boff[(kk % XBOX_K) / 16]);
            }
            if (XF16) {
              if (h == 0)
                mma_f16_z(t[gb][nt], A, bx.x, bx.y);
              else
                mma_f16(t[gb][nt], A, bx.x, bx.y);
            } else {
              if (h == 0)
                mma_bf16_z(t[gb][nt], A, bx.x, bx.y);
              else
                mma_bf16(t[gb][nt], A, bx.x, bx.y);
            }
          }
        }
      }
#pragma unroll
      for (int gb = 0; gb < GB; gb++) {
        const int blk = b0 + gb, j = blk / G::BPC, bb = blk % G::BPC;
        float2 d = decode_scales(sv[j][bb], SUBN);
        if (XF16 && FMT == 0) d.y *= 0.0625f;  // rows g+8 were decoded as 16q
        const float2 dg = make_float2(d.x, d.x), dh = make_float2(d.y, d.y);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
          acc[nt][0] = __ffma2_rn(make_float2(t[gb][nt][0], t[gb][nt][1]), dg, acc[nt][0]);
          acc[nt][1] = __ffma2_rn(make_float2(t[gb][nt][2], t[gb][nt][3]), dh, acc[nt][1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
}

template <int FMT, int NT>
__global__ void __launch_bounds__(THREADS, NT <= 2 ? 3 : 2)
    gemv_q_kernel(const __grid_constant__ CUtensorMap xmap, const GemvArgs a) {
  using G = Geo<FMT>;
  constexpr int BR = 8 * NT;  // padded batch rows
  constexpr bool XF16 = XMode<NT>::F16;
  constexpr int KCS = XF16 ? CS : BCS;           // chunks per stage
  constexpr int NSTG = XF16 ? STAGES : BSTAGES;  // ring depth
  constexpr int STG = XF16 ? G::STAGE : G::BSTG;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // the batch path's swizzled boxes need 1024-byte alignment
  uint8_t *smem = XF16 ? smem_raw
                       : reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t *stages = smem;
  uint16_t *xs = reinterpret_cast<uint16_t *>(smem + NSTG * STG);  // XF16 only
  float *red = reinterpret_cast<float *>(smem);  // reuses the stages after the main loop
  __shared__ __align__(8) uint64_t full[NSTG], empty[NSTG];
  __shared__ int s_exp[BR];
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x, s = blockIdx.y;
  // k-splits own whole stages (the chunk count is a multiple of CS)
  const int n_stages = a.n_chunks / KCS;
  const int st0 = (int)((long long)s * n_stages / a.S);
  const int n_iter = (int)((long long)(s + 1) * n_stages / a.S) - st0;
  const int c0 = st0 * KCS, nck = n_iter * KCS;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSTG; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CWARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == CWARPS) {
    // ---------------- producer: one bulk copy of CS records per stage (+ the
    // stage's x rows for large batches)
    if (lane == 0) {
      // the group's 8 tiles are 8 contiguous streams of (tile, chunk) units;
      // a stage holds CS units of each, tile-major
      const uint8_t *src = a.records + ((size_t)g * CWARPS * a.n_chunks + c0) * G::UNIT;
      const size_t tile_stride = (size_t)a.n_chunks * G::UNIT;
      constexpr uint32_t TB = KCS * G::UNIT;  // bytes of one tile in a stage
      constexpr uint32_t WB = CWARPS * TB;    // weight bytes of a stage
      auto copy_stage = [&](uint8_t *dst, int it, uint64_t *bar) {
#pragma unroll
        for (int t = 0; t < CWARPS; t++) bulk_g2s(dst + t * TB, src + t * tile_stride + (size_t)it * TB, TB, bar);
      };
      if (XF16) {
        for (int it = 0; it < n_iter; it++) {
          const int slot = it % NSTG;
          if (it >= NSTG && !mbar_wait(&empty[slot], ((it / NSTG) & 1) ^ 1)) atomicExch(a.err, 1);
          mbar_expect_tx(&full[slot], WB);
          copy_stage(stages + slot * STG, it, &full[slot]);
        }
      } else {
        // weights of the first stages before waiting for the kernel that
        // produces x; each stage's single arrival comes after its x boxes
        // (columns past K arrive as zeros)
        const int pre = min(NSTG, n_iter);
        for (int it = 0; it < pre; it++) {
          mbar_expect_tx_only(&full[it], WB);
          copy_stage(stages + it * STG, it, &full[it]);
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const uint32_t xbytes = (uint32_t)(G::NXB * a.B * XBOX_K * 2);
        for (int it = 0; it < n_iter; it++) {
          const int slot = it % NSTG;
          uint8_t *dst = stages + slot * STG;
          if (it >= NSTG) {
            if (!mbar_wait(&empty[slot], ((it / NSTG) & 1) ^ 1)) atomicExch(a.err, 1);
            mbar_expect_tx_only(&full[slot], WB);
            copy_stage(dst, it, &full[slot]);
          }
          const int kst = (c0 + it * KCS) * G::CH;
          mbar_expect_tx_only(&full[slot], xbytes);
#pragma unroll
          for (int xb = 0; xb < G::NXB; xb++)
            vxb::tc::tma_load_2d(dst + G::BWP + xb * XBOX_BYTES, &xmap, kst + xb * XBOX_K, 0, &full[slot]);
          mbar_arrive(&full[slot]);
        }
      }
    }
    asm volatile("griddepcontrol.launch_dependents;");
    __syncwarp();
    if (a.cluster) {
      // take part in the two cluster barriers of the reduction
      cluster_sync_all();
      cluster_sync_all();
    }
    return;
  }

  // ---------------- consumers
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const bool subnormal = (__ldg(a.hdr + 1) & TILED_FLAG_SUBNORMAL_SCALES) != 0;
  if (!XF16) {
    if (threadIdx.x < BR) s_exp[threadIdx.x] = 0;
  } else {
    const int k0 = c0 * G::CH, kc = nck * G::CH;
    const int nb = min(a.B, BR);
    // x[:, k0:k0+kc] (bf16) by 16-byte async copies of the live batch rows;
    // columns past K are zero-filled
    const int per_row = kc / 8;
    const int total = nb * per_row;
    for (int i = threadIdx.x; i < total; i += CWARPS * 32) {
      const int b = i / per_row, p = i % per_row;
      const int kk = k0 + p * 8;
      const bool ok = kk < a.K;
      cp_async16(xs + (size_t)b * a.xs_stride + p * 8, ok ? a.x + (size_t)b * a.K + kk : a.x, ok ? 16 : 0);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    consumer_sync();
    // per column: e with max|x| * 2^-e in [2^14, 2^15) (0 for an all-zero or
    // non-finite column)
    for (int b = warp; b < BR; b += CWARPS) {
      unsigned m = 0;
      if (b < nb) {
        const uint32_t *row = reinterpret_cast<const uint32_t *>(xs + (size_t)b * a.xs_stride);
        for (int i = lane; i < kc / 2; i += 32) {
          const uint32_t v = row[i];
          m = max(m, max(v & 0x7FFFu, (v >> 16) & 0x7FFFu));
        }
      }
      m = __reduce_max_sync(0xffffffffu, m);
      if (lane == 0) s_exp[b] = (m != 0 && m < 0x7F80u) ? max((int)(m >> 7), 1) - 127 - 14 : 0;
    }
    consumer_sync();
    // in place: bf16 x -> f16 x * 2^-e (exact)
    for (int i = threadIdx.x; i < total; i += CWARPS * 32) {
      const int b = i / per_row, p = i % per_row;
      uint4 *ptr = reinterpret_cast<uint4 *>(xs + (size_t)b * a.xs_stride + p * 8);
      uint4 v = *ptr;
      const int e = -s_exp[b];
      uint32_t *w = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
      for (int j = 0; j < 4; j++)
        w[j] = pack_f16x2(mul_pow2(__uint_as_float(w[j] << 16), e), mul_pow2(__uint_as_float(w[j] & 0xFFFF0000u), e));
      *ptr = v;
    }
  }
  consumer_sync();

  float2 acc[NT][2];  // [nt][row g | row g+8] x (batch column 2q, 2q+1)
  if (subnormal)
    consume_stages<FMT, NT, true>(a, stages, full, empty, xs, n_iter, acc);
  else
    consume_stages<FMT, NT, false>(a, stages, full, empty, xs, n_iter, acc);

  // every stage has been consumed and no copy is in flight: reuse the ring
  consumer_sync();
  {
    const int rl = warp * 16 + (lane >> 2);
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      const int b = nt * 8 + (lane & 3) * 2;
      const int e0 = s_exp[b], e1 = s_exp[b + 1];
      red[(size_t)b * ROWS_PER_CTA + rl] = mul_pow2(acc[nt][0].x, e0);
      red[(size_t)(b + 1) * ROWS_PER_CTA + rl] = mul_pow2(acc[nt][0].y, e1);
      red[(size_t)b * ROWS_PER_CTA + rl + 8] = mul_pow2(acc[nt][1].x, e0);
      red[(size_t)(b + 1) * ROWS_PER_CTA + rl + 8] = mul_pow2(acc[nt][1].y, e1);
    }
  }
  consumer_sync();

  const int row0 = g * ROWS_PER_CTA;
  const int nrows = min(ROWS_PER_CTA, a.N - row0);
  const int nel = a.B * ROWS_PER_CTA;
  if (a.S == 1) {
    for (int i = threadIdx.x; i < nel; i += CWARPS * 32) {
      const int b = i / ROWS_PER_CTA, r = i % ROWS_PER_CTA;
      if (r < nrows) epilogue_store(a, b, row0 + r, red[i]);
    }
    return;
  }
  if (a.cluster) {
    // the S k-splits of this row group form one cluster: every CTA sums a
    // slice of the outputs over the partials in the peers' shared memory, in
    // split order (deterministic), then the cluster waits until all reads are
    // done before any CTA exits
    __syncwarp();
    cluster_sync_all();
    // four consecutive outputs per thread and 16-byte distributed loads, the
    // S peers' loads all issued before the sum (nel and the slices are
    // multiples of 4)
    const int per = ((nel / 4 + a.S - 1) / a.S) * 4;
    const int i1 = min(nel, (s + 1) * per);
    cg::cluster_group cl = cg::this_cluster();
    for (int i = s * per + 4 * threadIdx.x; i < i1; i += 4 * CWARPS * 32) {
      float4 pv[kMaxClusterSplits];
#pragma unroll
      for (int ss = 0; ss < kMaxClusterSplits; ss++)
        if (ss < a.S) pv[ss] = *reinterpret_cast<const float4 *>(cl.map_shared_rank(red + i, (unsigned)ss));
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int ss = 0; ss < kMaxClusterSplits; ss++)
        if (ss < a.S) {
          v.x += pv[ss].x;
          v.y += pv[ss].y;
          v.z += pv[ss].z;
          v.w += pv[ss].w;
        }
      const int b = i / ROWS_PER_CTA, r = i % ROWS_PER_CTA;  // 4 rows of one batch column
      if (r < nrows) epilogue_store(a, b, row0 + r, v.x);
      if (r + 1 < nrows) epilogue_store(a, b, row0 + r + 1, v.y);
      if (r + 2 < nrows) epilogue_store(a, b, row0 + r + 2, v.z);
      if (r + 3 < nrows) epilogue_store(a, b, row0 + r + 3, v.w);
    }
    __syncwarp();
    cluster_sync_all();
    return;
  }
  const size_t NP = (size_t)a.NP;
  for (int i = threadIdx.x; i < nel; i += CWARPS * 32) {
    const int b = i / ROWS_PER_CTA, r = i % ROWS_PER_CTA;
    if (r < nrows) __stcg(a.ws + ((size_t)s * a.B + b) * NP + row0 + r, red[i]);
  }
  __threadfence();
  consumer_sync();
  if (threadIdx.x == 0) s_last = atomicAdd(a.counters + g, 1u) == (unsigned)(a.S - 1);
  consumer_sync();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < nel; i += CWARPS * 32) {
    const int b = i / ROWS_PER_CTA, r = i % ROWS_PER_CTA;
    if (r >= nrows) continue;
    // partials in split order; loads issued four at a time
    const float *src = a.ws + (size_t)b * NP + row0 + r;
    const size_t step = (size_t)a.B * NP;
    float v = 0.f;
    int ss = 0;
    for (; ss + 4 <= a.S; ss += 4) {
      const float p0 = __ldcg(src + ss * step), p1 = __ldcg(src + (ss + 1) * step);
      const float p2 = __ldcg(src + (ss + 2) * step), p3 = __ldcg(src + (ss + 3) * step);
      v += p0;
      v += p1;
      v += p2;
      v += p3;
    }
    for (; ss < a.S; ss++) v += __ldcg(src + ss * step);
    epilogue_store(a, b, row0 + r, v);
  }
  if (threadIdx.x == 0) a.counters[g] = 0u;
}

// ---------------------------------------------------------------------------
// Batch 1 (and Q4_0 up to batch 8): per-warp streams.
//
// Every warp owns one (16-row tile, k-part) and streams that contiguous run of
// units through its own ring of shared-memory stages with bulk copies issued
// by its lane 0; the first stages are requested before the wait for the
// kernel that produces x, so the weights stream while that kernel finishes.
// After the wait each warp copies the x columns of its k-part into shared
// memory (at batch 1 a private copy; for a batch, one copy per k-part shared
// by the CTA's warps of different tiles). Q4_0 codes are decoded to exact bf16
// values and multiplied with the bf16 activations as they are (no conversion
// pass, so a batch up to 8 is one MMA column per row); Q8_0 codes decode to
// f16 (one PRMT and one HSUB2 per two codes), so the warp converts its x
// columns to f16 scaled by 2^-e (max|x| * 2^-e in [2^14, 2^15), exact) -
// batch 1 only. The
// KQ warps of a CTA that share a tile add their partials through shared
// memory in warp order; with S > 1 the S CTAs of a cluster hold the other
// k-parts of the same tiles and add through distributed shared memory in CTA
// order. No global scratch, deterministic sums.
constexpr int SW_WARPS = 8;
constexpr int SW_THREADS = SW_WARPS * 32;
constexpr int SW_MAX_RING = 4;  // stages per warp ring

struct StreamArgs {
  const uint8_t *units;  // unit (tile 0, chunk 0)
  const uint32_t *hdr;
  const uint16_t *x;  // bf16 [B, K]
  void *y;
  const float *resid;  // optional f32 [B, N] added in the epilogue
  int *err;
  int N, K, B, n_chunks, y_dtype;
  int xs_stride;  // elements per batch row of one k-part's x columns
  int KQ, S;      // warps per tile inside a CTA, CTAs per tile (one cluster)
  int ring;       // stages in each warp's ring
  int wreg;       // shared-memory bytes of one warp's ring
  int xoff;       // offset of the x columns (KQ parts x B rows) behind the rings
};

__device__ __forceinline__ void store_out(const StreamArgs &a, int b, int row, float v) {
  const size_t o = (size_t)b * a.N + row;
  if (a.resid) v += __ldcg(a.resid + o);
  if (a.y_dtype == VXB_BF16)
    ((uint16_t *)a.y)[o] = f32_to_bf16_bits(v);
  else
    ((float *)a.y)[o] = v;
}

// acc[0] = rows g, acc[1] = rows g+8 of the warp's tile, batch columns
// (2q, 2q+1) with q = lane % 4.
template <int FMT, bool BAT, bool SUBN>
__device__ __forceinline__ void stream_consume(const StreamArgs &a, const uint8_t *src, uint8_t *ring, uint64_t *full,
                                               const uint16_t *xs, int n_iter, float2 (&acc)[2]) {
  using G = Geo<FMT>;
  constexpr uint32_t STB = CS * G::UNIT;
  const int lane = threadIdx.x & 31;
  acc[0] = acc[1] = make_float2(0.f, 0.f);
  const int B = BAT ? a.B : 1;
  const bool live = (lane >> 2) < B;  // the lanes whose B-operand column is a batch row
  const uint16_t *xl = xs + (BAT ? (lane >> 2) * a.xs_stride : 0) + (lane & 3) * 4;
  constexpr int BLK = CS * G::BPC;  // blocks per stage
  constexpr int GB = 4;             // blocks per group of independent accumulators
  for (int it = 0; it < n_iter; it++) {
    const int slot = it % a.ring;
    if (!mbar_wait(&full[slot], (it / a.ring) & 1)) atomicExch(a.err, 1);
    const uint8_t *st = ring + slot * STB;
    uint4 wv[CS];
    uint32_t sv[CS][G::BPC];
#pragma unroll
    for (int j = 0; j < CS; j++) {
      wv[j] = *reinterpret_cast<const uint4 *>(st + j * G::UNIT + lane * 16);
      const uint8_t *sp = st + j * G::UNIT + 512 + (lane >> 2) * G::BPC * 4;
      if (G::BPC == 2) {
        const uint2 t2 = *reinterpret_cast<const uint2 *>(sp);
        sv[j][0] = t2.x;
        sv[j][G::BPC - 1] = t2.y;
      } else {
        sv[j][0] = *reinterpret_cast<const uint32_t *>(sp);
      }
    }
    // the slot's data is in registers: refill it with stage it + ring
    __syncwarp();
    if (lane == 0 && it + a.ring < n_iter) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect_tx(&full[slot], STB);
      bulk_g2s(ring + slot * STB, src + (size_t)(it + a.ring) * STB, STB, &full[slot]);
    }
    const uint16_t *xk = xl + it * CS * G::CH;
#pragma unroll
    for (int b0 = 0; b0 < BLK; b0 += GB) {
      float t[GB][4];
#pragma unroll
      for (int h = 0; h < 2; h++) {
#pragma unroll
        for (int gb = 0; gb < GB; gb++) {
          const int blk = b0 + gb, j = blk / G::BPC, bb = blk % G::BPC;
          const uint32_t *wu = reinterpret_cast<const uint32_t *>(&wv[j]);
          uint32_t A[4];
          uint2 bx = make_uint2(0u, 0u);
          if (live) bx = *reinterpret_cast<const uint2 *>(xk + blk * 32 + h * 16);
          if (FMT == 0) {
            decode_q4_bf16(wu[bb * 2 + h], A);
            if (h == 0)
              mma_bf16_z(t[gb], A, bx.x, bx.y);
            else
              mma_bf16(t[gb], A, bx.x, bx.y);
          } else {
            decode_q8(wu[h * 2], wu[h * 2 + 1], A);
            if (h == 0)
              mma_f16_z(t[gb], A, bx.x, bx.y);
            else
              mma_f16(t[gb], A, bx.x, bx.y);
          }
        }
      }
#pragma unroll
      for (int gb = 0; gb < GB; gb++) {
        const int blk = b0 + gb, j = blk / G::BPC, bb = blk % G::BPC;
        const float2 d = decode_scales(sv[j][bb], SUBN);
        acc[0] = __ffma2_rn(make_float2(t[gb][0], t[gb][1]), make_float2(d.x, d.x), acc[0]);
        acc[1] = __ffma2_rn(make_float2(t[gb][2], t[gb][3]), make_float2(d.y, d.y), acc[1]);
      }
    }
  }
}

// BAT: a batch of 1..8 rows (Q4_0 only) with each k-part's x columns shared
// by the CTA's warps; otherwise batch 1 with a private copy per warp.
template <int FMT, bool BAT>
__global__ void __launch_bounds__(SW_THREADS) gemv_stream_kernel(const StreamArgs a) {
  static_assert(FMT == 0 || !BAT, "Q8_0 streams batch 1 only");
  using G = Geo<FMT>;
  constexpr uint32_t STB = CS * G::UNIT;  // one stage: CS units of one tile
  constexpr int SPAN = CS * G::CH;        // columns of one stage
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[SW_WARPS][SW_MAX_RING];
  constexpr int RC = BAT ? 8 : 1;           // batch columns kept per row
  __shared__ float red[SW_WARPS][16][RC];  // per-warp partials [row][batch column]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int B = BAT ? a.B : 1;
  const int RT = SW_WARPS / a.KQ;    // tiles per CTA
  const int tile = blockIdx.x * RT + warp / a.KQ;
  const int P = a.KQ * a.S;  // k-parts per tile
  const int part = blockIdx.y * a.KQ + warp % a.KQ;
  const int n_stages = a.n_chunks / CS;
  const int s0 = (int)((long long)part * n_stages / P);
  const int n_iter = (int)((long long)(part + 1) * n_stages / P) - s0;
  uint8_t *ring = smem + (size_t)warp * a.wreg;
  uint16_t *const xs = BAT ? reinterpret_cast<uint16_t *>(smem + a.xoff) + (size_t)(warp % a.KQ) * B * a.xs_stride
                           : reinterpret_cast<uint16_t *>(ring + (size_t)a.ring * STB);
  const uint8_t *src = a.units + ((size_t)tile * a.n_chunks + (size_t)s0 * CS) * G::UNIT;

  if (lane == 0) {
    for (int i = 0; i < a.ring; i++) mbar_init(&full[warp][i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // weights do not depend on the previous kernel: request them now
    const int pre = min(a.ring, n_iter);
    for (int it = 0; it < pre; it++) {
      mbar_expect_tx(&full[warp][it], STB);
      bulk_g2s(ring + it * STB, src + (size_t)it * STB, STB, &full[warp][it]);
    }
  }
  __syncwarp();
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const bool subnormal = (__ldg(a.hdr + 1) & TILED_FLAG_SUBNORMAL_SCALES) != 0;

  // ---- the x columns of this warp's k-part (shared by the RT warps of the
  // k-part when BAT): 16-byte asynchronous copies through the load/store path
  // and L2 only (the bulk-copy queue is busy with weights), zeros past K (K
  // and every part's first column are multiples of 32)
  {
    const int k0 = s0 * SPAN, n8 = n_iter * SPAN / 8;
    const int kv8 = max(0, min(n8, (a.K - k0) / 8));
    const int i0 = BAT ? (warp / a.KQ) * 32 + lane : lane, di = BAT ? SW_THREADS / a.KQ : 32;
    for (int b = 0; b < B; b++)
      for (int i = i0; i < n8; i += di) {
        uint16_t *dst = xs + (size_t)b * a.xs_stride + i * 8;
        if (i < kv8)
          cp_async16(dst, a.x + (size_t)b * a.K + k0 + i * 8, 16);
        else
          *reinterpret_cast<uint4 *>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  // the warps of one k-part share its x columns (KQ is uniform over the CTA)
  if (!BAT || a.KQ == SW_WARPS)
    __syncwarp();
  else
    __syncthreads();
  const int kr = n_iter * SPAN;
  int e = 0;
  if (FMT != 0) {
    // f16 operands: e with max|x| * 2^-e in [2^14, 2^15) (0 for all-zero or
    // non-finite x), then x * 2^-e in place
    unsigned m = 0;
    const uint32_t *row = reinterpret_cast<const uint32_t *>(xs);
    for (int i = lane; i < kr / 2; i += 32) {
      const uint32_t v = row[i];
      m = max(m, max(v & 0x7FFFu, (v >> 16) & 0x7FFFu));
    }
    m = __reduce_max_sync(0xffffffffu, m);
    e = (m != 0 && m < 0x7F80u) ? max((int)(m >> 7), 1) - 127 - 14 : 0;
    for (int p = lane; p < kr / 8; p += 32) {
      uint4 *ptr = reinterpret_cast<uint4 *>(xs) + p;
      uint4 v = *ptr;
      uint32_t *w = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
      for (int j = 0; j < 4; j++)
        w[j] = pack_f16x2(mul_pow2(__uint_as_float(w[j] << 16), -e), mul_pow2(__uint_as_float(w[j] & 0xFFFF0000u), -e));
      *ptr = v;
    }
    __syncwarp();
  }

  float2 acc[2];
  if (subnormal)
    stream_consume<FMT, BAT, true>(a, src, ring, full[warp], xs, n_iter, acc);
  else
    stream_consume<FMT, BAT, false>(a, src, ring, full[warp], xs, n_iter, acc);
  {
    const int r = lane >> 2, c = (lane & 3) * 2;
    if (RC > 1) {
      red[warp][r][c] = acc[0].x;
      red[warp][r][c + 1] = acc[0].y;
      red[warp][r + 8][c] = acc[1].x;
      red[warp][r + 8][c + 1] = acc[1].y;
    } else if (c == 0) {
      red[warp][r][0] = mul_pow2(acc[0].x, e);
      red[warp][r + 8][0] = mul_pow2(acc[1].x, e);
    }
  }
  __syncthreads();

  // ---- the KQ warps of each tile, in warp order; output i = (tile, row, column)
  const int nout = RT * 16 * B;
  float *cta_sum = reinterpret_cast<float *>(smem);  // the rings are free now
  for (int i = threadIdx.x; i < nout; i += SW_THREADS) {
    const int rt = i / (16 * B), rr = (i / B) % 16, b = i % B;
    float v = 0.f;
    for (int q = 0; q < a.KQ; q++) v += red[rt * a.KQ + q][rr][b];
    if (a.S == 1) {
      const int row = (blockIdx.x * RT + rt) * 16 + rr;
      if (row < a.N) store_out(a, b, row, v);
    } else {
      cta_sum[i] = v;
    }
  }
  if (a.S == 1) return;
  // ---- the S CTAs of the cluster hold the other k-parts: each sums a slice
  // of the outputs over the peers in CTA order; nobody exits before all reads
  // are done
  cluster_sync_all();
  cg::cluster_group cl = cg::this_cluster();
  const int per = (nout + a.S - 1) / a.S;
  const int i1 = min(nout, ((int)blockIdx.y + 1) * per);
  for (int i = (int)blockIdx.y * per + threadIdx.x; i < i1; i += SW_THREADS) {
    float v = 0.f;
    for (int ss = 0; ss < a.S; ss++) v += *cl.map_shared_rank(cta_sum + i, (unsigned)ss);
    const int rt = i / (16 * B), rr = (i / B) % 16, b = i % B;
    const int row = (blockIdx.x * RT + rt) * 16 + rr;
    if (row < a.N) store_out(a, b, row, v);
  }
  cluster_sync_all();
}

struct StreamPlan {
  int KQ = 0, S = 0, ring = 0, wreg = 0, xs_stride = 0;
  size_t smem = 0;
};

template <int FMT, bool BAT>
int stream_resident(size_t smem, int cluster, int sms) {
  static std::mutex mu;
  static std::map<std::pair<size_t, int>, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(smem, cluster);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  auto kfn = gemv_stream_kernel<FMT, BAT>;
  int n = 0;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) == cudaSuccess) {
    if (cluster <= 1) {
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, SW_THREADS, smem) == cudaSuccess) n = per_sm * sms;
    } else {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, cluster);
      cfg.blockDim = dim3(SW_THREADS);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 1;
      attr.val.clusterDim.y = cluster;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kfn, &cfg) == cudaSuccess) n = clusters * cluster;
    }
  }
  if (n < 1) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}

// Split of each tile's k range into KQ warps x S CTAs and the ring depth:
// minimise the busiest SM's stage count (CTAs spread evenly), inflated when
// fewer than 32 warps per SM hide the latency, plus the cost of a cluster
// reduction (about 1.5 us, some 30 stages of an SM's work) and of each wave
// beyond the first (its CTAs start streaming only when the first wave ends).
StreamPlan stream_plan(const vxb_ctx *ctx, const TiledGeom &g, int batch) {
  const int sms = ctx->num_sms > 0 ? ctx->num_sms : 148;
  const int n_stages = g.n_chunks / CS;
  const size_t stb = (size_t)CS * (512 + g.sc_per_tile);
  const int span = CS * g.chunk;
  StreamPlan best;
  double best_cost = 1e30;
  for (int KQ : {8, 4, 2, 1}) {
    for (int S : {1, 2, 4, 8}) {
      const int P = KQ * S;
      if (P > n_stages) continue;
      const int part_max = (n_stages + P - 1) / P;
      // batch 1: a private x copy behind each warp's ring; a batch: one copy
      // per k-part behind all rings, rows padded so that stride/2 = 8 (mod
      // 32) spreads the batch rows over the banks
      const int xs_stride = batch > 1 ? part_max * span + 16 : 0;
      const size_t xpriv = batch > 1 ? 0 : ((size_t)part_max * span * 2 + 127) / 128 * 128;
      const size_t xshared = (size_t)KQ * batch * xs_stride * 2;
      for (int ring = 2; ring <= SW_MAX_RING; ring++) {
        const int rg = std::min(ring, part_max);
        if (rg < ring && ring > 2) break;
        const size_t wreg = ((size_t)rg * stb + xpriv + 127) / 128 * 128;
        const size_t cta_sum = (size_t)(SW_WARPS / KQ) * 16 * batch * 4;
        const size_t smem = std::max((size_t)SW_WARPS * wreg + xshared, cta_sum);
        if (smem > 200 * 1024) continue;
        const int slots = g.fmt == VXB_Q8_0 ? stream_resident<1, false>(smem, S, sms)
                          : batch > 1      ? stream_resident<0, true>(smem, S, sms)
                                           : stream_resident<0, false>(smem, S, sms);
        if (slots < 1) continue;
        const int ctas = g.n_tiles / (SW_WARPS / KQ) * S;
        const int waves = (ctas + slots - 1) / slots;
        const double per_sm = std::min((double)ctas / sms, (double)slots / sms);
        const double wps = per_sm * SW_WARPS;
        const double load = (double)((ctas + sms - 1) / sms) * SW_WARPS * part_max;
        const double cost = load * (1.0 + std::max(0.0, (32.0 - wps) / 32.0)) + (S > 1 ? 30.0 : 0.0) +
                            40.0 * (waves - 1) - 0.5 * rg;
        if (cost < best_cost - 1e-9) {
          best_cost = cost;
          best.KQ = KQ;
          best.S = S;
          best.ring = rg;
          best.wreg = (int)wreg;
          best.xs_stride = xs_stride;
          best.smem = smem;
        }
      }
    }
  }
  return best;
}

template <int FMT, bool BAT>
int stream_launch_t(vxb_ctx *ctx, const StreamArgs &a, dim3 grid, size_t smem, cudaStream_t st, bool pdl) {
  auto kfn = gemv_stream_kernel<FMT, BAT>;
  static bool configured[64] = {false};
  const int dev = ctx->device & 63;
  if (!configured[dev]) {
    VXB_CUDA_TRY(ctx, cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(SW_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  if (a.S > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = a.S;
    attr[na].val.clusterDim.z = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  VXB_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kfn, a));
  return VXB_OK;
}

// Batches the per-warp stream kernel takes: Q4_0 multiplies bf16 activations
// directly, one MMA column per row up to 8 (past batch 4 the group-CTA kernel
// is faster on 7B shapes); Q8_0 rescales its f16 activations per k-part and
// runs batch 1 only.
bool stream_eligible(int fmt, int batch) { return batch == 1 || (fmt == VXB_Q4_0 && batch <= 4); }

// y = W x (+ resid) through the per-warp stream kernel: batch 1, or Q4_0 up
// to batch 8 (one B-operand column per activation row).
int stream_gemv(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x, int batch,
                int y_dtype, void *d_y, const float *d_resid, int *d_err, cudaStream_t st, bool pdl, const char *who) {
  const TiledGeom g = tiled_geom(fmt, N, K);
  const StreamPlan p = stream_plan(ctx, g, batch);
  if (p.KQ == 0) return set_error(ctx, VXB_EINVAL, "%s: no launch plan fits N=%d K=%d", who, N, K);
  StreamArgs a;
  const uint8_t *base = (const uint8_t *)d_tiled;
  a.units = base + g.codes_off;
  a.hdr = (const uint32_t *)base;
  a.x = d_x;
  a.y = d_y;
  a.resid = d_resid;
  a.err = d_err;
  a.N = N;
  a.K = K;
  a.B = batch;
  a.n_chunks = g.n_chunks;
  a.y_dtype = y_dtype;
  a.xs_stride = p.xs_stride;
  a.KQ = p.KQ;
  a.S = p.S;
  a.ring = p.ring;
  a.wreg = p.wreg;
  a.xoff = SW_WARPS * p.wreg;
  const dim3 grid(g.n_tiles / (SW_WARPS / p.KQ), p.S);
  if (fmt == VXB_Q8_0) return stream_launch_t<1, false>(ctx, a, grid, p.smem, st, pdl);
  return batch > 1 ? stream_launch_t<0, true>(ctx, a, grid, p.smem, st, pdl)
                   : stream_launch_t<0, false>(ctx, a, grid, p.smem, st, pdl);
}

size_t smem_bytes_t(int fmt, int NT, int batch, int xs_stride) {
  const size_t stage = fmt == VXB_Q4_0 ? Geo<0>::STAGE : Geo<1>::STAGE;
  const size_t bstage = fmt == VXB_Q4_0 ? Geo<0>::BSTG : Geo<1>::BSTG;
  const size_t red = (size_t)8 * NT * ROWS_PER_CTA * 4;
  // + 1024 bytes to align the batch path's ring for the swizzled boxes
  if (NT > 1) return std::max((size_t)BSTAGES * bstage, red) + 1024;
  return std::max((size_t)STAGES * stage, red) + (size_t)std::min(batch, 8 * NT) * xs_stride * 2;
}

// Tensor map of the activations x [B, K] bf16 for the batch path: boxes of
// 64 columns x B rows, 128-byte swizzle, columns past K read as zero.
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

int x_tensor_map(vxb_ctx *ctx, const uint16_t *x, int B, int K, CUtensorMap *map) {
  const EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return set_error(ctx, VXB_ECUDA, "vxb_gemv_q: cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)B};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)XBOX_K, (cuuint32_t)B};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VXB_OK;
}

int xs_stride_for(int kc_max) { return kc_max + 16; }  // stride/2 = 8 (mod 32): conflict-free 8-byte loads

// Largest k-range of one split: splits own whole stages of CS chunks, so a
// split spans at most ceil(stages / S) stages (the kernel's split bounds).
int kc_max_for(const TiledGeom &g, int S) {
  const int n_stages = g.n_chunks / CS;
  return (n_stages + S - 1) / S * CS * g.chunk;
}

// CTAs of an instantiation that can be resident on the whole GPU at a
// shared-memory size: per-SM occupancy x SMs for plain launches, the largest
// number of co-resident clusters x S for clusters of S CTAs (cached).
template <int FMT, int NT>
int resident_t(size_t smem, int cluster, int sms) {
  static std::mutex mu;
  static std::map<std::pair<size_t, int>, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(smem, cluster);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  auto kfn = gemv_q_kernel<FMT, NT>;
  int n = 0;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) == cudaSuccess) {
    if (cluster <= 1) {
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, THREADS, smem) == cudaSuccess) n = per_sm * sms;
    } else {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, cluster);
      cfg.blockDim = dim3(THREADS);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 1;
      attr.val.clusterDim.y = cluster;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kfn, &cfg) == cudaSuccess) n = clusters * cluster;
    }
  }
  if (n < 1) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}

int resident(int fmt, int NT, size_t smem, int cluster, int sms) {
  if (fmt == VXB_Q4_0) {
    switch (NT) {
      case 1: return resident_t<0, 1>(smem, cluster, sms);
      case 2: return resident_t<0, 2>(smem, cluster, sms);
      case 3: return resident_t<0, 3>(smem, cluster, sms);
      default: return resident_t<0, 4>(smem, cluster, sms);
    }
  }
  switch (NT) {
    case 1: return resident_t<1, 1>(smem, cluster, sms);
    case 2: return resident_t<1, 2>(smem, cluster, sms);
    case 3: return resident_t<1, 3>(smem, cluster, sms);
    default: return resident_t<1, 4>(smem, cluster, sms);
  }
}

template <int FMT, int NT>
int launch_t(vxb_ctx *ctx, const GemvArgs &a, dim3 grid, size_t smem, cudaStream_t st, bool pdl) {
  auto kfn = gemv_q_kernel<FMT, NT>;
  CUtensorMap xmap;  // the batch path's activation boxes (unused for batch <= 8)
  memset(&xmap, 0, sizeof(xmap));
  if (NT > 1)
    if (int rc = x_tensor_map(ctx, a.x, a.B, a.K, &xmap)) return rc;
  static bool configured[64] = {false};
  const int dev = ctx->device & 63;
  if (!configured[dev]) {
    VXB_CUDA_TRY(ctx, cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  if (a.cluster) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = grid.y;
    attr[na].val.clusterDim.z = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  VXB_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kfn, xmap, a));
  return VXB_OK;
}


// ---------------------------------------------------------------------------
// Batches 9-32: tcgen05 skinny GEMM (opt-in: VXB_GEMV_TCGEN05=1).
//
// A CTA owns one 128-row group (8 tiles) and a k-range of whole weight stages
// (qps quads of 4 chunks of each tile). Per 64-column step the group's codes become the A
// operand of tcgen05.mma in tensor memory: exact small integers as bf16,
// written by the decode warp of each TMEM lane quadrant q (tiles 2q, 2q+1)
// with tcgen05.st.16x256b, whose register layout (thread t: lanes t/4 and
// t/4+8, columns 2(t%4) and 2(t%4)+1) is the m16n8k16 A fragment the tiled
// units already hold, with the units' k permutation lining the fragment up
// with the matrix columns. x is the 128-byte-swizzled K-major B operand [NB
// rows x 64 columns] (rows past the batch and columns past K zero), copied by
// one warp with 16-byte cp.async through the load/store path: a TMA load
// would queue behind the CTA's ~200 KB of weight bulk copies (measured: ~6 us
// per x stage instead of ~1). Each
// 32-column block accumulates into its own NB TMEM columns (two M=128 x N=NB
// x K=16 MMAs), so the epilogue multiplies the block's f32 sums by the f16
// block scales (acc += d * D, in block order) as the mma.sync kernels do: the
// scales never round into an operand.
//
// The weights of a stage (qps quads of 4 chunks of each of the 8 tiles, 18 or
// 37 KB) arrive by one 3-D TMA load over the tiled layout viewed as [tiles]
// [chunks][unit words]: issuing eight bulk copies of 1-2 KB per stage from one
// thread held a CTA to ~7 GB/s.
// Warps: 0 weight producer (issued before the wait for the previous kernel),
// 1 TMEM allocation and MMA issue, 2 x producer,
// 3-6 decode (lane quadrants 3, 0, 1, 2), 7-10 epilogue (quadrants 3, 0, 1, 2).
// S > 1 CTAs of a row group form a cluster and add their partial sums through
// distributed shared memory in CTA order.
constexpr int TC_THREADS = 352;
constexpr int TC_AR = 4;   // A slots in TMEM (32 columns = 64 bf16 codes per row each)
constexpr int TC_DR = 2;   // accumulator slots (2 blocks x NB columns each)
constexpr int TC_SR = 8;   // scale slots in shared memory (one step each)
constexpr int TC_XR = 8;   // x stages (one step each)
constexpr int TC_XLAG = 4;  // x steps in flight (cp.async groups) before the oldest is published
constexpr int TC_MAX_WR = 24;
constexpr uint32_t TC_COLS = 256, TC_ACOL = 0, TC_DCOL = 128;
constexpr int TC_SMEM_MAX = 225 * 1024;  // dynamic shared memory (the barriers are static)

struct TcArgs {
  const uint8_t *units;  // unit (tile 0, chunk 0)
  const uint32_t *hdr;
  const uint16_t *x;  // bf16 [B, K]
  void *y;
  const float *resid;  // optional f32 [B, N]
  int *err;
  int N, K, B, n_chunks, y_dtype;
  int wr;     // weight stages in the ring
  int qps;    // quads (4 chunks) per weight stage
  int n_wst;  // weight stages over the padded k range (the last may reach past it: zeros)
  int S;      // CTAs per row group (cluster along y)
};

template <int FMT>
struct TcGeo {
  static constexpr int UNIT = Geo<FMT>::UNIT;
  static constexpr int SPQ = FMT == 0 ? 4 : 2;  // 64-column steps per quad of 4 chunks
  __host__ __device__ static constexpr int wsb(int qps) { return 8 * 4 * qps * UNIT; }  // one weight stage
};

template <int NB>
struct TcSmem {
  static constexpr int XB = NB * 128;  // one x stage: NB rows x 64 bf16
  static constexpr int X_OFF = 0;
  static constexpr int W_OFF = TC_XR * XB;
  __host__ __device__ static size_t sc_off(int wsb, int wr) { return (size_t)W_OFF + (size_t)wsb * wr; }
  __host__ __device__ static size_t red_off(int wsb, int wr) { return sc_off(wsb, wr) + (size_t)TC_SR * 2 * 128 * 4; }
  __host__ __device__ static size_t bytes(int wsb, int wr, int S) {
    return red_off(wsb, wr) + (S > 1 ? (size_t)NB * 128 * 4 : 0) + 1024;  // + 1024: base alignment
  }
};

__device__ __forceinline__ void tmem_st_16x256b_x4(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

template <int NB>
__device__ __forceinline__ void tmem_ld_nb(uint32_t taddr, float (&v)[NB]) {
  if constexpr (NB == 32)
    vxb::tc::tmem_ld32(taddr, v);
  else
    tmem_ld16(taddr, v);
}

// bounded wait that records a failure once and then stops waiting
__device__ __forceinline__ void tc_wait(uint64_t *bar, uint32_t parity, bool &ok, int *err) {
  if (ok && !mbar_wait(bar, parity)) {
    ok = false;
    atomicExch(err, 1);
  }
}

// the same for all lanes of a warp, with a warp-uniform outcome (the lanes
// stay converged for the elected arrivals)
__device__ __forceinline__ void tc_wait_warp(uint64_t *bar, uint32_t parity, bool &ok, int *err) {
  bool mine = ok;
  if (mine && !mbar_wait(bar, parity)) mine = false;
  const bool all = __all_sync(0xffffffffu, mine);
  if (ok && !all && (threadIdx.x & 31) == 0) atomicExch(err, 1);
  ok = all;
}

// one arrival per warp: the lanes' prior accesses are ordered before it by
// the warp barrier (32 arrivals on one mbarrier serialize for ~1 us)
__device__ __forceinline__ void warp_arrive(uint64_t *bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// The 16x256b.x4 registers of one tile for one 64-column step: k16 step s
// holds {row g: k 4q..4q+1, row g: 4q+2..4q+3, row g+8: 4q..4q+1, row g+8:
// 4q+2..4q+3} = fragment pairs {a0a1, a4a5, a2a3, a6a7}.
template <int FMT>
__device__ __forceinline__ void tc_decode_tile(const uint8_t *u0, const uint8_t *u1, int lane, uint32_t (&r)[16]) {
  const uint4 c0 = *reinterpret_cast<const uint4 *>(u0 + lane * 16);
  if (FMT == 0) {
    const uint32_t w[4] = {c0.x, c0.y, c0.z, c0.w};
#pragma unroll
    for (int s = 0; s < 4; s++) {
      uint32_t A[4];
      decode_q4_bf16(w[s], A);
      r[4 * s + 0] = A[0];
      r[4 * s + 1] = A[2];
      r[4 * s + 2] = A[1];
      r[4 * s + 3] = A[3];
    }
  } else {
    const uint4 c1 = *reinterpret_cast<const uint4 *>(u1 + lane * 16);
    const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
    for (int s = 0; s < 4; s++) {
      uint32_t A[4];
      decode_q8_bf16(w[2 * s], w[2 * s + 1], A);
      r[4 * s + 0] = A[0];
      r[4 * s + 1] = A[2];
      r[4 * s + 2] = A[1];
      r[4 * s + 3] = A[3];
    }
  }
}

// one x step [NB rows x 64 columns] into a 128-byte-swizzled stage: 16-byte
// chunk c of row r at r * 128 + ((c ^ (r % 8)) * 16); zeros past B and K
template <int NB>
__device__ __forceinline__ void tc_x_step(const TcArgs &a, uint8_t *dst, int k0, int lane) {
#pragma unroll
  for (int i = 0; i < NB * 8 / 32; i++) {
    const int idx = lane + 32 * i, r = idx >> 3, c = idx & 7;
    const bool in = r < a.B && k0 + c * 8 < a.K;
    const uint16_t *src = in ? a.x + (size_t)r * a.K + k0 + c * 8 : a.x;
    cp_async16(dst + r * 128 + ((c ^ (r & 7)) << 4), src, in ? 16 : 0);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int FMT, int NB>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap wmap, const TcArgs a) {
  using TG = TcGeo<FMT>;
  using SM = TcSmem<NB>;
  constexpr int UNIT = TG::UNIT;
  const int WSTEPS = a.qps * TG::SPQ, WSB = TG::wsb(a.qps), TBYTES = 4 * a.qps * UNIT;  // TBYTES: one tile's part
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t *xring = sm + SM::X_OFF;
  uint8_t *wring = sm + SM::W_OFF;
  float *sc = reinterpret_cast<float *>(sm + SM::sc_off(WSB, a.wr));  // [TC_SR][2][128]
  float *red = reinterpret_cast<float *>(sm + SM::red_off(WSB, a.wr));  // [NB][128] (S > 1)
  __shared__ __align__(8) uint64_t wfull[TC_MAX_WR], wempty[TC_MAX_WR], xfull[TC_XR], xempty[TC_XR];
  __shared__ __align__(8) uint64_t afull[TC_AR], aempty[TC_AR], dfull[TC_DR], dempty[TC_DR];
  __shared__ __align__(8) uint64_t sfull[TC_SR], sempty[TC_SR], mdone;
  __shared__ uint32_t tmem_base_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = blockIdx.x;
  const int ws0 = (int)((long long)blockIdx.y * a.n_wst / a.S);
  const int nws = (int)((long long)(blockIdx.y + 1) * a.n_wst / a.S) - ws0;
  const int nsteps = nws * WSTEPS;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(TC_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.wr; i++) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], 4);
    }
    for (int i = 0; i < TC_XR; i++) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xempty[i], 1);
    }
    for (int i = 0; i < TC_AR; i++) {
      mbar_init(&afull[i], 4);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < TC_DR; i++) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], 4);
    }
    for (int i = 0; i < TC_SR; i++) {
      mbar_init(&sfull[i], 4);
      mbar_init(&sempty[i], 4);
    }
    mbar_init(&mdone, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  vxb::tc::tc_fence_before();
  __syncthreads();
  vxb::tc::tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  asm volatile("griddepcontrol.launch_dependents;");
  bool ok = true;

  if (warp == 0) {
    // ---------------- weights: one TMA box [8 tiles][4 qps chunks][unit] per
    // stage. The whole warp waits (a lone spinning lane beside 31 lanes parked
    // at a warp barrier woke ~1 us after its barrier completed); lane 0 issues.
    for (int ws = 0; ws < nws; ws++) {
      const int slot = ws % a.wr;
      if (ws >= a.wr) tc_wait_warp(&wempty[slot], ((ws / a.wr) - 1) & 1, ok, a.err);
      if (!ok) break;
      if (lane == 0) {
        mbar_expect_tx(&wfull[slot], WSB);
        vxb::tc::tma_load_3d(wring + (size_t)slot * WSB, &wmap, 0, (ws0 + ws) * 4 * a.qps, grp * 8, &wfull[slot]);
      }
      __syncwarp();
    }
    // copies still in flight finish before the CTA exits
    for (int ws = max(0, nws - a.wr); ws < nws; ws++) {
      bool dr = true;
      tc_wait_warp(&wfull[ws % a.wr], (ws / a.wr) & 1, dr, a.err);
    }
  } else if (warp == 2) {
    // ---------------- x: per step 16-byte cp.async of all 32 lanes (one
    // commit group); step st - TC_XLAG is published once its group landed
    // (cp.async.wait_group, then a proxy fence: the MMA reads it through the
    // async proxy)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int k0 = ws0 * WSTEPS * 64;
    int issued = 0;
    for (int st = 0; st < nsteps; st++) {
      const int slot = st % TC_XR;
      if (st >= TC_XR) tc_wait_warp(&xempty[slot], ((st / TC_XR) - 1) & 1, ok, a.err);
      if (!ok) break;
      tc_x_step<NB>(a, xring + slot * SM::XB, k0 + st * 64, lane);
      issued = st + 1;
      if (st >= TC_XLAG) {
        asm volatile("cp.async.wait_group %0;" ::"n"(TC_XLAG) : "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        warp_arrive(&xfull[(st - TC_XLAG) % TC_XR]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int st = max(0, issued - TC_XLAG); st < issued; st++) warp_arrive(&xfull[st % TC_XR]);
  } else if (warp == 1) {
    // ---------------- MMA: per step, blocks b = 0, 1 into accumulator slot
    // columns [b * NB, b * NB + NB), two K=16 MMAs each; the warp waits, lane 0
    // issues
    constexpr uint32_t ID = vxb::tc::idesc_bf16(128, NB, false);
    for (int st = 0; st < nsteps; st++) {
      const int as = st % TC_AR, xs = st % TC_XR, ds = st % TC_DR;
      tc_wait_warp(&afull[as], (st / TC_AR) & 1, ok, a.err);
      tc_wait_warp(&xfull[xs], (st / TC_XR) & 1, ok, a.err);
      if (st >= TC_DR) tc_wait_warp(&dempty[ds], ((st / TC_DR) - 1) & 1, ok, a.err);
      if (!ok) break;
      vxb::tc::tc_fence_after();
      if (lane == 0) {
        const uint32_t xa = smem_u32(xring + xs * SM::XB);
#pragma unroll
        for (int b = 0; b < 2; b++)
#pragma unroll
          for (int k = 0; k < 2; k++)
            vxb::tc::umma_bf16_ts(tmem + TC_DCOL + ds * 2 * NB + b * NB, tmem + TC_ACOL + as * 32 + (2 * b + k) * 8,
                                  vxb::tc::sw128_desc(xa + (2 * b + k) * 32, 16, 1024), ID, k);
        vxb::tc::umma_commit(&aempty[as]);
        vxb::tc::umma_commit(&xempty[xs]);
        vxb::tc::umma_commit(&dfull[ds]);
      }
      __syncwarp();
    }
    if (lane == 0) vxb::tc::umma_commit(&mdone);  // every MMA issued above has completed
    __syncwarp();
    bool dr = true;
    tc_wait_warp(&mdone, 0, dr, a.err);
  } else if (warp <= 6) {
    // ---------------- decode: TMEM lane quadrant q = warp % 4, tiles 2q, 2q+1
    const int q = warp & 3;
    const bool subn = (__ldg(a.hdr + 1) & TILED_FLAG_SUBNORMAL_SCALES) != 0;
    // this lane's scales go to the epilogue row 32q + lane: tile 2q + lane/16,
    // row pair (lane % 16) % 8, half (lane % 16) / 8
    const int je = 2 * q + (lane >> 4), pi = (lane & 15) & 7, ph = (lane & 15) >> 3;
    for (int st = 0; st < nsteps; st++) {
      const int ws = st / WSTEPS, sub = st % WSTEPS, wslot = ws % a.wr;
      const int as = st % TC_AR, ss = st % TC_SR;
      if (sub == 0) tc_wait_warp(&wfull[wslot], (ws / a.wr) & 1, ok, a.err);
      if (st >= TC_AR) tc_wait_warp(&aempty[as], ((st / TC_AR) - 1) & 1, ok, a.err);
      if (st >= TC_SR) tc_wait_warp(&sempty[ss], ((st / TC_SR) - 1) & 1, ok, a.err);
      if (!ok) break;
      vxb::tc::tc_fence_after();
      const uint8_t *stg = wring + (size_t)wslot * WSB;
      // Q4_0: unit `sub` of the tile (4 k16 steps); Q8_0: units 2 sub, 2 sub + 1 (2 each)
      const int u0 = FMT == 0 ? sub : 2 * sub;
      const uint8_t *t0 = stg + (2 * q) * TBYTES + u0 * UNIT;
      const uint8_t *t1 = stg + (2 * q + 1) * TBYTES + u0 * UNIT;
      uint32_t r0[16], r1[16];
      tc_decode_tile<FMT>(t0, t0 + UNIT, lane, r0);
      tc_decode_tile<FMT>(t1, t1 + UNIT, lane, r1);
      float s0, s1;
      {
        const uint8_t *ue = stg + je * TBYTES + u0 * UNIT + 512;
        uint32_t w0, w1;
        if (FMT == 0) {
          const uint2 t = *reinterpret_cast<const uint2 *>(ue + pi * 8);
          w0 = t.x;
          w1 = t.y;
        } else {
          w0 = *reinterpret_cast<const uint32_t *>(ue + pi * 4);
          w1 = *reinterpret_cast<const uint32_t *>(ue + UNIT + pi * 4);
        }
        const float2 d0 = decode_scales(w0, subn), d1 = decode_scales(w1, subn);
        s0 = ph ? d0.y : d0.x;
        s1 = ph ? d1.y : d1.x;
      }
      if (sub == WSTEPS - 1) warp_arrive(&wempty[wslot]);  // the warp's reads of the stage are done
      const uint32_t ta = tmem + TC_ACOL + as * 32 + ((uint32_t)(32 * q) << 16);
      tmem_st_16x256b_x4(ta, r0);
      tmem_st_16x256b_x4(ta + (16u << 16), r1);
      sc[(ss * 2 + 0) * 128 + 32 * q + lane] = s0;
      sc[(ss * 2 + 1) * 128 + 32 * q + lane] = s1;
      vxb::tc::tmem_wait_st();
      vxb::tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&afull[as]);
        mbar_arrive(&sfull[ss]);
      }
    }
  } else {
    // ---------------- epilogue: row 32q + lane of the group, all NB columns
    const int q = warp & 3;
    const int row = grp * 128 + 32 * q + lane;
    float acc[NB];
#pragma unroll
    for (int n = 0; n < NB; n++) acc[n] = 0.f;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int st = 0; st < nsteps; st++) {
      const int ds = st % TC_DR, ss = st % TC_SR;
      tc_wait_warp(&dfull[ds], (st / TC_DR) & 1, ok, a.err);
      tc_wait_warp(&sfull[ss], (st / TC_SR) & 1, ok, a.err);
      if (!ok) break;
      vxb::tc::tc_fence_after();
      float v0[NB], v1[NB];
      const uint32_t td = tmem + TC_DCOL + ds * 2 * NB + ((uint32_t)(32 * q) << 16);
      tmem_ld_nb<NB>(td, v0);
      tmem_ld_nb<NB>(td + NB, v1);
      vxb::tc::tmem_wait_ld();
      vxb::tc::tc_fence_before();
      const float s0 = sc[(ss * 2 + 0) * 128 + 32 * q + lane];
      const float s1 = sc[(ss * 2 + 1) * 128 + 32 * q + lane];
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&dempty[ds]);
        mbar_arrive(&sempty[ss]);
      }
#pragma unroll
      for (int n = 0; n < NB; n++) acc[n] = fmaf(s1, v1[n], fmaf(s0, v0[n], acc[n]));
    }
    if (a.S == 1) {
      if (row < a.N)
#pragma unroll
        for (int n = 0; n < NB; n++) {
          if (n >= a.B) break;
          const size_t o = (size_t)n * a.N + row;
          float v = acc[n];
          if (a.resid) v += __ldcg(a.resid + o);
          if (a.y_dtype == VXB_BF16)
            ((uint16_t *)a.y)[o] = f32_to_bf16_bits(v);
          else
            ((float *)a.y)[o] = v;
        }
    } else {
#pragma unroll
      for (int n = 0; n < NB; n++) red[n * 128 + 32 * q + lane] = acc[n];
    }
  }

  if (a.S > 1) {
    // ---- the S CTAs of the row group: CTA c sums a slice of the outputs over
    // the peers in CTA order; nobody exits before all reads are done
    cluster_sync_all();
    cg::cluster_group cl = cg::this_cluster();
    const int nout = a.B * 128;
    const int per = (nout + a.S - 1) / a.S;
    const int i1 = min(nout, ((int)blockIdx.y + 1) * per);
    asm volatile("griddepcontrol.wait;" ::: "memory");  // before the first global write of this thread
    for (int i = (int)blockIdx.y * per + threadIdx.x; i < i1; i += TC_THREADS) {
      const int n = i >> 7, rr = i & 127;
      float v = 0.f;
      for (int s = 0; s < a.S; s++) v += *cl.map_shared_rank(red + n * 128 + rr, (unsigned)s);
      const int row = grp * 128 + rr;
      if (row < a.N) {
        const size_t o = (size_t)n * a.N + row;
        if (a.resid) v += __ldcg(a.resid + o);
        if (a.y_dtype == VXB_BF16)
          ((uint16_t *)a.y)[o] = f32_to_bf16_bits(v);
        else
          ((float *)a.y)[o] = v;
      }
    }
    cluster_sync_all();
  }
  vxb::tc::tc_fence_before();
  __syncthreads();
  vxb::tc::tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_COLS));
}

struct TcPlan {
  int S = 0, wr = 0, qps = 0, n_wst = 0;
  size_t smem = 0;
};

template <int FMT, int NB>
int tc_resident(size_t smem, int cluster, int sms) {
  static std::mutex mu;
  static std::map<std::pair<size_t, int>, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(smem, cluster);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  auto kfn = gemv_tc_kernel<FMT, NB>;
  int n = 0;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_MAX) == cudaSuccess) {
    if (cluster <= 1) {
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, TC_THREADS, smem) == cudaSuccess)
        n = per_sm * sms;
    } else {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, cluster);
      cfg.blockDim = dim3(TC_THREADS);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 1;
      attr.val.clusterDim.y = cluster;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kfn, &cfg) == cudaSuccess) n = clusters * cluster;
    }
  }
  if (n < 1) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}

// k-splits S and ring depth: the time is the larger of the whole weight
// stream at the HBM rate and the busiest SM's share at a per-SM rate of about
// 120 GB/s, plus about 0.5 us for a cluster reduction and 1 us per extra
// wave. When the CTAs need two per SM, each ring is sized so that two fit.
template <int FMT, int NB>
TcPlan tc_plan_t(const vxb_ctx *ctx, const TiledGeom &g) {
  const int sms = ctx->num_sms > 0 ? ctx->num_sms : 148;
  const int n_quads = g.n_chunks / 4;
  TcPlan best;
  double best_cost = 1e30;
  for (int qps : {2, 1})
  for (int S : {1, 2, 4, 8}) {
    const int wsb = TcGeo<FMT>::wsb(qps);
    const int n_wst = (n_quads + qps - 1) / qps;
    if (S > n_wst) break;
    const int ctas = g.n_groups * S;
    const int per_cta = (n_wst + S - 1) / S;
    const int per_sm = std::min(2, (ctas + sms - 1) / sms);
    const size_t budget = per_sm == 1 ? TC_SMEM_MAX : 112 * 1024;
    const size_t fixed = TcSmem<NB>::bytes(wsb, 0, S);
    if (fixed + 2 * (size_t)wsb > budget) continue;
    const int wr = std::min({TC_MAX_WR, per_cta, (int)((budget - fixed) / wsb)});
    if (wr < 1) continue;
    const size_t smem = TcSmem<NB>::bytes(wsb, wr, S);
    const int slots = tc_resident<FMT, NB>(smem, S, sms);
    if (slots < 1) continue;
    const int waves = (ctas + slots - 1) / slots;
    const double t_hbm = (double)ctas * per_cta * wsb / 6.5e6;
    const double t_sm = (double)((ctas + sms - 1) / sms) * per_cta * wsb / 1.2e5;
    const double cost = std::max(t_hbm, t_sm) + (S > 1 ? 0.5 : 0.0) + 1.0 * (waves - 1);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best.S = S;
      best.wr = wr;
      best.qps = qps;
      best.n_wst = n_wst;
      best.smem = smem;
    }
  }
  return best;
}

// The tiled units as a 3-D u32 tensor [tiles][chunks][unit words]: boxes of
// 8 tiles x 4 qps chunks x one unit (chunks past the padded k range read as
// zero bytes: codes with scale 0).
int weights_tensor_map(vxb_ctx *ctx, const uint8_t *units, const TiledGeom &g, int qps, CUtensorMap *map) {
  const EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return set_error(ctx, VXB_ECUDA, "vxb_gemv_q: cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {(cuuint64_t)(g.unit / 4), (cuuint64_t)g.n_chunks, (cuuint64_t)g.n_tiles};
  cuuint64_t strides[2] = {(cuuint64_t)g.unit, (cuuint64_t)g.n_chunks * g.unit};
  cuuint32_t box[3] = {(cuuint32_t)(g.unit / 4), (cuuint32_t)(4 * qps), 8};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t *>(units), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: weight tensor map failed (%d)", (int)r);
  return VXB_OK;
}

template <int FMT, int NB>
int tc_launch_t(vxb_ctx *ctx, const TcArgs &a0, const TiledGeom &g, cudaStream_t st, bool pdl) {
  auto kfn = gemv_tc_kernel<FMT, NB>;
  const TcPlan p = tc_plan_t<FMT, NB>(ctx, g);
  if (p.S == 0) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: no tensor-core launch plan fits N=%d K=%d", a0.N, a0.K);
  CUtensorMap wmap;
  if (int rc = weights_tensor_map(ctx, a0.units, g, p.qps, &wmap)) return rc;
  static bool configured[64] = {false};
  const int dev = ctx->device & 63;
  if (!configured[dev]) {
    VXB_CUDA_TRY(ctx, cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_MAX));
    configured[dev] = true;
  }
  TcArgs a = a0;
  a.wr = p.wr;
  a.qps = p.qps;
  a.n_wst = p.n_wst;
  a.S = p.S;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g.n_groups, p.S);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  if (p.S > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = p.S;
    attr[na].val.clusterDim.z = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  VXB_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kfn, wmap, a));
  return VXB_OK;
}

// y = W x (+ resid) for batches 9..32 through the tcgen05 kernel.
int tc_gemv(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x, int batch, int y_dtype,
            void *d_y, const float *d_resid, int *d_err, cudaStream_t st, bool pdl) {
  const TiledGeom g = tiled_geom(fmt, N, K);
  TcArgs a = {};
  const uint8_t *base = (const uint8_t *)d_tiled;
  a.units = base + g.codes_off;
  a.hdr = (const uint32_t *)base;
  a.x = d_x;
  a.y = d_y;
  a.resid = d_resid;
  a.err = d_err;
  a.N = N;
  a.K = K;
  a.B = batch;
  a.n_chunks = g.n_chunks;
  a.y_dtype = y_dtype;
  if (fmt == VXB_Q4_0)
    return batch <= 16 ? tc_launch_t<0, 16>(ctx, a, g, st, pdl) : tc_launch_t<0, 32>(ctx, a, g, st, pdl);
  return batch <= 16 ? tc_launch_t<1, 16>(ctx, a, g, st, pdl) : tc_launch_t<1, 32>(ctx, a, g, st, pdl);
}

// The tensor-core kernel is exact and parity-tested but not yet faster than
// the group-CTA kernel (a fixed ~0.8 us per 64-column step), so batches 9-32
// take it only when the process sets VXB_GEMV_TCGEN05=1.
bool tc_enabled() {
  static const bool on = [] {
    const char *v = getenv("VXB_GEMV_TCGEN05");
    return v && v[0] == '1';
  }();
  return on;
}

bool tc_eligible(int batch) { return tc_enabled() && batch >= 9 && batch <= 32; }

}  // namespace

namespace vxb {

size_t gemv_smem_bytes(int fmt, int N, int K, int batch, int S) {
  const TiledGeom g = tiled_geom(fmt, N, K);
  const int NT = (batch + 7) / 8;
  const int kc_max = kc_max_for(g, S);
  return smem_bytes_t(fmt, NT, batch, xs_stride_for(kc_max));
}

GemvPlan gemv_plan(const vxb_ctx *ctx, int fmt, int N, int K, int batch) {
  const TiledGeom g = tiled_geom(fmt, N, K);
  const int row_groups = g.n_groups;
  const int sms = ctx->num_sms > 0 ? ctx->num_sms : 148;
  // Each CTA streams at a rate set by its stage ring, so the run time is the
  // number of CTA waves times the duration of one CTA (proportional to 1/S):
  // pick the split count that minimises waves/S, with a small cost per wave.
  // Up to kMaxClusterSplits splits reduce through distributed shared memory
  // inside one cluster; more splits reduce through global memory, which costs
  // a few more round trips. Resident CTAs per SM come from the occupancy
  // calculator.
  int best = 0;
  double best_cost = 1e30;
  const int smax = std::min(32, g.n_chunks / CS);
  for (int S = 1; S <= smax; S++) {
    const size_t sm = gemv_smem_bytes(fmt, N, K, batch, S);
    if (sm > 200 * 1024) continue;
    const int slots = resident(fmt, (batch + 7) / 8, sm, S > 1 && S <= kMaxClusterSplits ? S : 1, sms);
    if (slots < 1) continue;
    const int waves = (row_groups * S + slots - 1) / slots;
    const double cost = (double)waves / S + 0.03 * waves + (S > kMaxClusterSplits ? 0.05 : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = S;
    }
  }
  if (best == 0) best = smax;  // nothing fits: the launch reports the shared-memory need
  GemvPlan p;
  p.S = best;
  p.cluster = best > 1 && best <= kMaxClusterSplits;
  p.pdl = true;
  return p;
}

int gemv_launch(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x, int batch,
                int y_dtype, void *d_y, const float *d_resid, void *stream, const GemvPlan *plan_override) {
  if (fmt != VXB_Q4_0 && fmt != VXB_Q8_0) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: unknown format %d", fmt);
  if (N <= 0 || K <= 0 || K % 32) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: bad shape N=%d K=%d", N, K);
  if (batch < 1 || batch > 32) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: batch %d outside 1..32", batch);
  if (y_dtype != VXB_F32 && y_dtype != VXB_BF16) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: y_dtype must be F32 or BF16");
  if (!d_tiled || !d_x || !d_y) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: null pointer");
  if (((uintptr_t)d_tiled) % 256) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: tiled weights must be 256-byte aligned");
  if (((uintptr_t)d_x) % 16) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: activations must be 16-byte aligned");
  if (int rc = use_device(ctx)) return rc;
  if (tc_eligible(batch) && !plan_override) {
    if (int rc = ws_reserve(ctx, 0, 0)) return rc;  // device error word
    return tc_gemv(ctx, fmt, d_tiled, N, K, d_x, batch, y_dtype, d_y, d_resid, ctx->d_err, (cudaStream_t)stream, true);
  }
  if (stream_eligible(fmt, batch) && !plan_override) {
    if (int rc = ws_reserve(ctx, 0, 0)) return rc;  // device error word
    return stream_gemv(ctx, fmt, d_tiled, N, K, d_x, batch, y_dtype, d_y, d_resid, ctx->d_err, (cudaStream_t)stream,
                       true, "vxb_gemv_q");
  }
  const TiledGeom g = tiled_geom(fmt, N, K);
  GemvPlan p = plan_override ? *plan_override : gemv_plan(ctx, fmt, N, K, batch);
  const int NT = (batch + 7) / 8;
  const int row_groups = g.n_groups;
  const int NP = (N + 15) / 16 * 16;  // row stride of the split-K partials
  const size_t ws_bytes = p.S > 1 ? (size_t)p.S * batch * NP * sizeof(float) : 0;
  if (int rc = ws_reserve(ctx, ws_bytes, (size_t)row_groups)) return rc;
  GemvArgs a;
  const uint8_t *base = (const uint8_t *)d_tiled;
  a.records = base + g.codes_off;
  a.hdr = (const uint32_t *)base;
  a.x = d_x;
  a.y = d_y;
  a.resid = d_resid;
  a.ws = (float *)ctx->ws;
  a.counters = ctx->counters;
  a.err = ctx->d_err;
  a.N = N;
  a.K = K;
  a.B = batch;
  a.NP = NP;
  a.n_chunks = g.n_chunks;
  a.S = p.S;
  a.cluster = p.cluster && p.S > 1 && p.S <= kMaxClusterSplits;
  a.y_dtype = y_dtype;
  const int kc_max = kc_max_for(g, p.S);
  a.xs_stride = xs_stride_for(kc_max);
  const size_t smem = smem_bytes_t(fmt, NT, batch, a.xs_stride);
  if (smem > 200 * 1024) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: split plan needs %zu bytes of shared memory", smem);
  dim3 grid(row_groups, p.S);
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  if (fmt == VXB_Q4_0) {
    switch (NT) {
      case 1: rc = launch_t<0, 1>(ctx, a, grid, smem, st, p.pdl); break;
      case 2: rc = launch_t<0, 2>(ctx, a, grid, smem, st, p.pdl); break;
      case 3: rc = launch_t<0, 3>(ctx, a, grid, smem, st, p.pdl); break;
      default: rc = launch_t<0, 4>(ctx, a, grid, smem, st, p.pdl); break;
    }
  } else {
    switch (NT) {
      case 1: rc = launch_t<1, 1>(ctx, a, grid, smem, st, p.pdl); break;
      case 2: rc = launch_t<1, 2>(ctx, a, grid, smem, st, p.pdl); break;
      case 3: rc = launch_t<1, 3>(ctx, a, grid, smem, st, p.pdl); break;
      default: rc = launch_t<1, 4>(ctx, a, grid, smem, st, p.pdl); break;
    }
  }
  return rc;
}

}  // namespace vxb

VXB_API int vxb_gemv_q(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x, int batch,
                       int y_dtype, void *d_y, void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_gemv_q: null context");
  return gemv_launch(ctx, fmt, d_tiled, N, K, d_x, batch, y_dtype, d_y, nullptr, stream, nullptr);
}

// ---------------------------------------------------------------------------
// GEMV without device allocation.
//
// vxb_gemv_q keeps its split-K partial sums, reduction counters and error word
// in the context workspace, which it grows with cudaMalloc on first use. Some
// callers cannot allow that: an embedding runtime that owns all device memory
// through its own arena, a caller that must not add allocations while other
// work holds a fixed memory budget, or code paths where a cudaMalloc would
// synchronize the device. vxb_gemv_q_static computes the same product with
// that scratch in the fixed array below instead. The caller still provides
// the weights, activations and output. Every GPU that loads the library holds
// the array (8 MiB of partials + 64 KiB of counters + the error word) until
// the process exits. All calls on a device share it, and it keeps the last
// call's contents: the counters are cleared before each launch, and calls that
// overlap on the GPU (different streams without ordering) race on it.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kStaticPartialBytes = (size_t)8 << 20;  // f32 split-K partials
constexpr int kStaticCounters = 16384;                   // one per 128-row group
constexpr size_t kStaticBytes = kStaticPartialBytes + (size_t)kStaticCounters * 4 + 256;

__device__ __align__(256) uint8_t g_static_scratch[kStaticBytes];

std::mutex g_static_mu;
uint8_t *g_static_addr[64] = {nullptr};

// Device address of g_static_scratch on the context's device (resolved once
// per device with that device current; the symbol's name in host code is a
// host-side stand-in, not a device address).
int static_scratch(vxb_ctx *ctx, uint8_t **out) {
  if (ctx->device < 0 || ctx->device >= 64) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q_static: device %d", ctx->device);
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_addr[ctx->device]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaGetSymbolAddress(g_static_scratch)");
    g_static_addr[ctx->device] = (uint8_t *)p;
  }
  *out = g_static_addr[ctx->device];
  return VXB_OK;
}

}  // namespace

VXB_API int vxb_gemv_q_static(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x,
                              int batch, int y_dtype, void *d_y, void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_gemv_q_static: null context");
  if (fmt != VXB_Q4_0 && fmt != VXB_Q8_0) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q_static: unknown format %d", fmt);
  if (N <= 0 || K <= 0 || K % 32) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q_static: bad shape N=%d K=%d", N, K);
  if (batch < 1 || batch > 32) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q_static: batch %d outside 1..32", batch);
  if (y_dtype != VXB_F32 && y_dtype != VXB_BF16)
    return set_error(ctx, VXB_EINVAL, "vxb_gemv_q_static: y_dtype must be F32 or BF16");
  if (!d_tiled || !d_x || !d_y) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q_static: null pointer");
  if (((uintptr_t)d_tiled) % 256 || ((uintptr_t)d_x) % 16)
    return set_error(ctx, VXB_EINVAL, "vxb_gemv_q_static: weights must be 256-byte and activations 16-byte aligned");
  const TiledGeom g = tiled_geom(fmt, N, K);
  const int NP = (N + 15) / 16 * 16;  // row stride of the split-K partials
  const size_t per_split = (size_t)batch * NP * sizeof(float);
  const int row_groups = g.n_groups;
  // the fixed array must hold the partials of at least two k-splits
  if (per_split * 2 > kStaticPartialBytes || row_groups > kStaticCounters)
    return set_error(ctx, VXB_EINVAL,
                     "vxb_gemv_q_static: batch * N = %d * %d exceeds the static scratch limit "
                     "(batch * round_up(N, 16) <= %zu)",
                     batch, N, kStaticPartialBytes / (2 * sizeof(float)));
  if (int rc = use_device(ctx)) return rc;
  uint8_t *base = nullptr;
  if (int rc = static_scratch(ctx, &base)) return rc;
  if (tc_eligible(batch))  // the tensor-core kernel needs no scratch beyond the error word
    return tc_gemv(ctx, fmt, d_tiled, N, K, d_x, batch, y_dtype, d_y, nullptr,
                   (int *)(base + kStaticPartialBytes + (size_t)kStaticCounters * 4), (cudaStream_t)stream, false);
  if (stream_eligible(fmt, batch))  // the per-warp stream kernel needs no scratch beyond the error word
    return stream_gemv(ctx, fmt, d_tiled, N, K, d_x, batch, y_dtype, d_y, nullptr,
                       (int *)(base + kStaticPartialBytes + (size_t)kStaticCounters * 4), (cudaStream_t)stream, false,
                       "vxb_gemv_q_static");
  GemvPlan p = gemv_plan(ctx, fmt, N, K, batch);
  p.S = std::max(1, std::min<int>(p.S, (int)(kStaticPartialBytes / per_split)));
  GemvArgs a;
  const uint8_t *wb = (const uint8_t *)d_tiled;
  a.records = wb + g.codes_off;
  a.hdr = (const uint32_t *)wb;
  a.x = d_x;
  a.y = d_y;
  a.resid = nullptr;
  a.ws = (float *)base;
  a.counters = (unsigned *)(base + kStaticPartialBytes);
  a.err = (int *)(base + kStaticPartialBytes + (size_t)kStaticCounters * 4);
  a.N = N;
  a.K = K;
  a.B = batch;
  a.NP = NP;
  a.n_chunks = g.n_chunks;
  a.S = p.S;
  a.cluster = p.cluster && p.S > 1 && p.S <= kMaxClusterSplits;
  a.y_dtype = y_dtype;
  const int kc_max = kc_max_for(g, p.S);
  a.xs_stride = xs_stride_for(kc_max);
  const int NT = (batch + 7) / 8;
  const size_t smem = smem_bytes_t(fmt, NT, batch, a.xs_stride);
  if (smem > 200 * 1024) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q_static: plan needs %zu bytes of shared memory", smem);
  cudaStream_t st = (cudaStream_t)stream;
  // counters must start at zero (a previous call that stopped early could have left them set)
  VXB_CUDA_TRY(ctx, cudaMemsetAsync(a.counters, 0, (size_t)row_groups * 4, st));
  dim3 grid(row_groups, p.S);
  if (fmt == VXB_Q4_0) {
    switch (NT) {
      case 1: return launch_t<0, 1>(ctx, a, grid, smem, st, false);
      case 2: return launch_t<0, 2>(ctx, a, grid, smem, st, false);
      case 3: return launch_t<0, 3>(ctx, a, grid, smem, st, false);
      default: return launch_t<0, 4>(ctx, a, grid, smem, st, false);
    }
  }
  switch (NT) {
    case 1: return launch_t<1, 1>(ctx, a, grid, smem, st, false);
    case 2: return launch_t<1, 2>(ctx, a, grid, smem, st, false);
    case 3: return launch_t<1, 3>(ctx, a, grid, smem, st, false);
    default: return launch_t<1, 4>(ctx, a, grid, smem, st, false);
  }
}
