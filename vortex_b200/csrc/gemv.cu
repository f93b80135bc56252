// K1: decode dequant-GEMV / skinny GEMM over tiled Q4_0 / Q8_0 weights.
//
//   y[b, n] = sum_k deq(W)[n, k] * x[b, k]     (b < batch <= 32)
//
// Replaces weight_only_matmul (src/quantize.rs:845-852, = dequantize then
// matmul_f64 890-902) and the matmul of Linear::forward
// (src/transformer.rs:332-352) at decode batch sizes.
//
// Two kernels (the tcgen05 kernel for batches 9-32 is in gemv_tc.cu, opt-in):
//  * gemv_stream_kernel - batch 1, and Q4_0 batches 2-4: every warp streams
//    one (16-row tile, k-part) through its own ring of bulk copies (see the
//    comment at the kernel).
//  * gemv_q_kernel - the other batches, the group-CTA design below.
//
// Group-CTA design (HBM-bound streaming):
//  * A CTA owns one 128-row group (8 sixteen-row tiles, one per consumer warp)
//    and a k-range. The tiled layout stores every (tile, k-chunk) as one
//    contiguous unit of codes and scales, and a tile's chunks back to back,
//    so a producer warp moves a stage (CS units of each of the 8 tiles) with 8
//    cp.async.bulk copies into a ring of shared-memory stages (one mbarrier
//    per stage with a transaction count).
//  * Consumer warps read their tile's codes with one 16-byte LDS per lane per
//    chunk (the slice is the lane's m16n8k16 A fragments) and turn them into
//    exact integers: for batch <= 8 f16 (Q4_0 nibbles by LOP3 with the f16
//    magic 1024 and one HSUB2 per two codes; Q8_0 bytes, stored as q+128, by
//    one PRMT with the magic byte and one HSUB2 per two codes), for larger
//    batches bf16.
//  * Batch <= 8: the activations of the CTA's k-range are staged once as f16,
//    each batch column multiplied by a power of two 2^-e chosen from its
//    largest magnitude (max |x| * 2^-e in [2^14, 2^15)), so the bf16 -> f16
//    conversion is exact for every element within 2^-28 of the column maximum
//    and nothing overflows; the f32 result is multiplied back by 2^e. Larger
//    batches carry their unchanged bf16 x slice in every stage as 2-D TMA
//    boxes with a 128-byte swizzle.
//  * mma.m16n8k16 (f32 accumulate) forms the per-block dot products; the
//    per-(row, block) f16 scale multiplies that f32 block partial with packed
//    f32x2 FMAs, so scales never round into the operands.
//  * Split-K across CTAs with a deterministic reduction: the splits of a row
//    group form a cluster and add through distributed shared memory in split
//    order, or (more than 8 splits) each CTA writes its f32 partial and the
//    last CTA of a row group (counter in global memory) sums the partials in
//    split order; the counter is returned to zero.
//  * The producer issues weight copies before any dependency on the kernel
//    that produces x, so under programmatic dependent launch the weight stream
//    overlaps the producer kernel's tail. Every mbarrier wait is bounded
//    (clock64); a timeout sets the context's device error word and the kernel
//    runs to completion.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>

#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gemv.h"
#include "gemv_common.h"
#include "tc_common.h"
#include "tiled_layout.h"
#include "vxb_internal.h"

using namespace vxb;
namespace cg = cooperative_groups;

namespace {

// Activations: batches up to 8 (XF16) stage the split's x once as f16 scaled
// per batch column by 2^-e; larger batches carry an unchanged bf16 x slice in
// every stage (no prologue, shared memory independent of K).
template <int NT>
struct XMode {
  static constexpr bool F16 = NT == 1;
};

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
// Batch 1, and Q4_0 batches 2-4 (routing: stream_eligible): per-warp streams.
// The kernel handles Q4_0 batches up to 8; past 4 the group kernel is faster.
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
// batch 1 only. The KQ warps of a CTA that share a tile add their partials
// through shared memory in warp order; with S > 1 the S CTAs of a cluster hold the other
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
  int slot = 0;      // it % ring, kept without a division
  uint32_t ph = 0u;  // (it / ring) & 1
  for (int it = 0; it < n_iter; it++) {
    if (!mbar_wait(&full[slot], ph)) atomicExch(a.err, 1);
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
    if (++slot == a.ring) {
      slot = 0;
      ph ^= 1u;
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
  static std::atomic<bool> configured[64];  // kernel attributes set on this device (zero-initialized)
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
  static std::atomic<bool> configured[64];  // kernel attributes set on this device (zero-initialized)
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
  if (gemv_tc_eligible(fmt, N, batch) && !plan_override) {
    if (int rc = ws_reserve(ctx, 0, 0)) return rc;  // device error word
    return gemv_tc(ctx, fmt, d_tiled, N, K, d_x, batch, y_dtype, d_y, d_resid, ctx->d_err, (cudaStream_t)stream, true);
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

constexpr size_t kStaticErrOff = kStaticPartialBytes + (size_t)kStaticCounters * 4;  // the error word

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

// Split count of the group kernel inside vxb_gemv_q_static: the array holds
// at most kStaticPartialBytes / per_split partial sets.
int static_splits(int planned, size_t per_split) {
  return std::max(1, std::min<int>(planned, (int)(kStaticPartialBytes / per_split)));
}

}  // namespace

namespace vxb {

// The error word of vxb_gemv_q_static's array on `device`, or null while no
// static call has resolved the array there (then nothing can have set it).
int *static_error_word(int device) {
  if (device < 0 || device >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_static_mu);
  return g_static_addr[device] ? (int *)(g_static_addr[device] + kStaticErrOff) : nullptr;
}

// The same word, resolving the array's address first (device made current by the caller).
int static_error_word_resolve(vxb_ctx *ctx, int **out) {
  uint8_t *base = nullptr;
  if (int rc = static_scratch(ctx, &base)) return rc;
  *out = (int *)(base + kStaticErrOff);
  return VXB_OK;
}

}  // namespace vxb

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
  if (gemv_tc_eligible(fmt, N, batch))  // the tensor-core kernel needs no scratch beyond the error word
    return gemv_tc(ctx, fmt, d_tiled, N, K, d_x, batch, y_dtype, d_y, nullptr,
                   (int *)(base + kStaticErrOff), (cudaStream_t)stream, false);
  if (stream_eligible(fmt, batch))  // the per-warp stream kernel needs no scratch beyond the error word
    return stream_gemv(ctx, fmt, d_tiled, N, K, d_x, batch, y_dtype, d_y, nullptr,
                       (int *)(base + kStaticErrOff), (cudaStream_t)stream, false, "vxb_gemv_q_static");
  GemvPlan p = gemv_plan(ctx, fmt, N, K, batch);
  p.S = static_splits(p.S, per_split);
  GemvArgs a;
  const uint8_t *wb = (const uint8_t *)d_tiled;
  a.records = wb + g.codes_off;
  a.hdr = (const uint32_t *)wb;
  a.x = d_x;
  a.y = d_y;
  a.resid = nullptr;
  a.ws = (float *)base;
  a.counters = (unsigned *)(base + kStaticPartialBytes);
  a.err = (int *)(base + kStaticErrOff);
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

VXB_API int vxb_gemv_plan_info(vxb_ctx *ctx, int fmt, int N, int K, int batch, int is_static, int *kernel,
                               int *splits, int *cluster) {
  if (!ctx || !kernel || !splits || !cluster) return set_error(ctx, VXB_EINVAL, "vxb_gemv_plan_info: null argument");
  if (fmt != VXB_Q4_0 && fmt != VXB_Q8_0) return set_error(ctx, VXB_EINVAL, "vxb_gemv_plan_info: unknown format %d", fmt);
  if (N <= 0 || K <= 0 || K % 32 || batch < 1 || batch > 32)
    return set_error(ctx, VXB_EINVAL, "vxb_gemv_plan_info: bad shape N=%d K=%d batch=%d", N, K, batch);
  if (int rc = use_device(ctx)) return rc;
  const TiledGeom g = tiled_geom(fmt, N, K);
  if (gemv_tc_eligible(fmt, N, batch)) {
    *kernel = 2;
    *splits = gemv_tc_splits(ctx, fmt, N, K, batch);
    *cluster = *splits > 1;
    return VXB_OK;
  }
  if (stream_eligible(fmt, batch)) {
    const StreamPlan p = stream_plan(ctx, g, batch);
    *kernel = 0;
    *splits = p.S;
    *cluster = p.S > 1;
    return VXB_OK;
  }
  GemvPlan p = gemv_plan(ctx, fmt, N, K, batch);
  if (is_static) p.S = static_splits(p.S, (size_t)batch * ((N + 15) / 16 * 16) * sizeof(float));
  *kernel = 1;
  *splits = p.S;
  *cluster = p.cluster && p.S > 1 && p.S <= kMaxClusterSplits;
  return VXB_OK;
}
