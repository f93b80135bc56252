// K2: prefill GEMM over quantized weights on the tcgen05 tensor cores.
//
//   Y[m, n] = sum_k X[m, k] * deq(W)[n, k]   (+ R[m, n])      X bf16, W Q4_0/Q8_0
//
// Replaces weight_only_matmul (src/quantize.rs:845-852, dequantize then
// matmul_f64 890-902) and Linear::forward (src/transformer.rs:332-352) for
// many rows (prefill).
//
// The block scale multiplies each weight: w = q * d with q at most 4 (Q4_0)
// or 8 (Q8_0) bits and d an f16, so w carries at most 15 / 19 significant
// bits. Each weight is split once per call into bf16 terms, t0 = bf16(w),
// t1 = bf16(w - t0) (and t2 = bf16(w - t0 - t1) for Q8_0), whose sum is w
// exactly. The GEMM then runs sum_t X * t^T into one f32 accumulator:
//  * CTA tile 128 rows of X x 256 rows of W, k in blocks of 64; a stage is
//    one (k block, term) pair, X 16 KB + the term's 32 KB, in a 4-deep ring,
//    loaded by TMA with 128-byte swizzle (no multicast; X is read once per
//    term, from L2);
//  * one thread issues tcgen05.mma (M=128, N=256, K=16; bf16 -> f32), four per
//    stage, into one of two TMEM partials (256 columns each, 4 k blocks =
//    256 k per partial, every term), and releases each stage with
//    tcgen05.commit;
//  * persistent CTAs, one per SM, walk the tiles (the m blocks of an n block
//    consecutively); the TMA and MMA warps run on into the next tile while
//    the epilogue warps write the previous one;
//  * eight epilogue warps (one output row and 128 columns per thread) add each partial
//    (tcgen05.ld) to the row's f32 sums in registers with round-to-nearest
//    adds, so the long K reduction keeps f32 accuracy (the tensor core's own
//    accumulation runs over 256 k at most) while the tensor core fills the
//    other partial; then they write Y (f32 or bf16) with the optional
//    residual.
// Every mbarrier wait is bounded; a timeout sets the context's device error
// word and the kernel runs to completion.
#include <algorithm>
#include <atomic>
#include <cuda.h>
#include <cuda_fp16.h>

#include <mutex>

#include "gemm.h"
#include "tc_common.h"
#include "tiled_layout.h"
#include "vxb_internal.h"

using namespace vxb;
using namespace vxb::tc;

namespace {

constexpr int BM = 128, BN = 256, BK = 64;
// k stages accumulated inside one TMEM partial before the epilogue adds it to
// the f32 row sums (256 columns of k per tensor-core accumulation)
constexpr int DRAIN = 4;
constexpr int THREADS = 320;  // warp 0: TMA, warp 1: MMA, warps 2-9: epilogue
constexpr int EPI_WARPS = 8;  // two per TMEM lane quadrant, one per 128-column half
constexpr int A_BYTES = BM * BK * 2;          // 16 KB
constexpr int B_BYTES = BN * BK * 2;          // 32 KB per weight term
constexpr uint32_t TMEM_COLS = 2 * BN;        // two stage partials

template <int TERMS>
struct GemmGeo {
  // a stage is one (k block, weight term) pair: the X tile and one term's
  // W tile, so the ring holds four stages whatever the term count (with all
  // terms of a k block in one stage, 128x256 tiles left room for two)
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (227 * 1024 - 1024) / STAGE_BYTES;
  static constexpr int SMEM_ALLOC = STAGES * STAGE_BYTES + 1024;
};
static_assert(GemmGeo<3>::SMEM_ALLOC <= 227 * 1024, "shared memory");

struct GemmArgs {
  void *y;
  const float *resid;
  int *err;
  int M, N, K, y_dtype;
};

template <int TERMS>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_terms_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw,
                      const GemmArgs a) {
  constexpr int STAGE_BYTES = GemmGeo<TERMS>::STAGE_BYTES;
  constexpr int STAGES = GemmGeo<TERMS>::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], pfull[2], pfree[2];
  __shared__ uint32_t tmem_base_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (a.K + BK - 1) / BK;
  // persistent: tiles blockIdx.x, + gridDim.x, ...; the m blocks of one n
  // block are consecutive (concurrent CTAs share W tiles in L2)
  const int mt = (a.M + BM - 1) / BM, ntile = mt * ((a.N + BN - 1) / BN);
  const int ngrp = (nk + DRAIN - 1) / DRAIN;  // TMEM partial groups per tile

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < STAGES; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pfree[i], EPI_WARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int ig = 0;  // stage count over all tiles of this CTA
      for (int tile = blockIdx.x; tile < ntile; tile += gridDim.x) {
        const int m0 = (tile % mt) * BM, n0 = (tile / mt) * BN;
        for (int it = 0; it < nk * TERMS; it++, ig++) {
          const int kb = it / TERMS, t = it % TERMS;
          const int st = ig % STAGES;
          if (ig >= STAGES) wait_or_flag(&empty[st], ((ig / STAGES) - 1) & 1, a.err);
          uint8_t *base = sm + st * STAGE_BYTES;
          mbar_expect_tx(&full[st], STAGE_BYTES);
          tma_load_2d(base, &tx, kb * BK, m0, &full[st]);
          // the terms are stacked [TERMS * N, K]: term t of rows n0.. at row t * N + n0
          tma_load_2d(base + A_BYTES, &tw, kb * BK, t * a.N + n0, &full[st]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issue: stage kb accumulates into TMEM partial kb % 2
    if (lane == 0) {
      constexpr uint32_t ID = idesc_bf16(BM, BN, false);
      int ig = 0, g0 = 0;  // stage and partial-group counts over all tiles of this CTA
      for (int tile = blockIdx.x; tile < ntile; tile += gridDim.x, g0 += ngrp)
      for (int it = 0; it < nk * TERMS; it++, ig++) {
        const int kb = it / TERMS, u = it % TERMS;
        const int st = ig % STAGES, grp = g0 + kb / DRAIN, pb = grp & 1;
        const bool first = kb % DRAIN == 0 && u == 0;
        const bool last = (kb % DRAIN == DRAIN - 1 || kb == nk - 1) && u == TERMS - 1;
        wait_or_flag(&full[st], (ig / STAGES) & 1, a.err);
        if (first && grp >= 2) wait_or_flag(&pfree[pb], ((grp >> 1) - 1) & 1, a.err);
        tc_fence_after();
        const uint32_t sa = smem_u32(sm + st * STAGE_BYTES);
        const uint32_t td = tmem + pb * BN;
#pragma unroll
        for (int t = 0; t < BK / 16; t++)
          umma_bf16(td, sw128_desc(sa + t * 32, 16, 1024), sw128_desc(sa + A_BYTES + t * 32, 16, 1024), ID,
                    (!first || t > 0) ? 1u : 0u);
        umma_commit(&empty[st]);
        if (last) umma_commit(&pfull[pb]);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: warp w owns TMEM lanes 32 * (w % 4) .. +31
    // and columns [128 * half, 128 * half + 128) of the tile; each partial is
    // added in f32 (round to nearest) to the row's sums
    const int q = warp & 3, half = (warp - 2) >> 2;
    int g0 = 0;  // partial-group count over all tiles of this CTA
    for (int tile = blockIdx.x; tile < ntile; tile += gridDim.x, g0 += ngrp) {
    const int m0 = (tile % mt) * BM, n0 = (tile / mt) * BN;
    const int row = m0 + q * 32 + lane;
    float acc[128];
#pragma unroll
    for (int i = 0; i < 128; i++) acc[i] = 0.f;
    for (int gi = 0; gi < ngrp; gi++) {
      const int grp = g0 + gi, pb = grp & 1;
      wait_or_flag(&pfull[pb], (grp >> 1) & 1, a.err);
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 128 / 32; c++) {
        float v[32];
        tmem_ld32(tmem + pb * BN + half * 128 + ((uint32_t)(q * 32) << 16) + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i++) acc[c * 32 + i] += v[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfree[pb]);
    }
    if (row < a.M) {
#pragma unroll
      for (int c = 0; c < 128 / 32; c++) {
        const int col0 = n0 + half * 128 + c * 32;
        if (col0 >= a.N) break;
        const size_t o = (size_t)row * a.N + col0;
        const int nv = min(32, a.N - col0);
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = acc[c * 32 + i];
        if (a.resid)
          for (int i = 0; i < nv; i++) v[i] += a.resid[o + i];
        if (a.y_dtype == VXB_BF16) {
          uint16_t *y = (uint16_t *)a.y + o;
          if (nv == 32 && (o % 8) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 w;
              w.x = pack_bf16(v[i], v[i + 1]);
              w.y = pack_bf16(v[i + 2], v[i + 3]);
              w.z = pack_bf16(v[i + 4], v[i + 5]);
              w.w = pack_bf16(v[i + 6], v[i + 7]);
              *reinterpret_cast<uint4 *>(y + i) = w;
            }
          } else {
            for (int i = 0; i < nv; i++) y[i] = f32_to_bf16_bits(v[i]);
          }
        } else {
          float *y = (float *)a.y + o;
          if (nv == 32 && (o % 4) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4 *>(y + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          } else {
            for (int i = 0; i < nv; i++) y[i] = v[i];
          }
        }
      }
    }
    }  // tile
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
}

// One thread per (row, 32-element block): w = q * d rebuilt from the tiled
// layout, written as `terms` bf16 parts [terms][N, K] summing to w.
__global__ void dequant_terms_kernel(const uint8_t *__restrict__ tiled, TiledGeom g, int terms,
                                     uint16_t *__restrict__ out) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int nbk = g.K / 32;
  if (idx >= (size_t)g.N * nbk) return;
  const int r = (int)(idx / nbk), b = (int)(idx % nbk);
  const int t = r / 16, ri = r % 16;
  const int bpc = g.chunk / 32;
  const bool subnormal = (reinterpret_cast<const uint32_t *>(tiled)[1] & TILED_FLAG_SUBNORMAL_SCALES) != 0;
  const uint32_t sbits =
      (*reinterpret_cast<const uint32_t *>(tiled + tiled_scales_at(g, t, b / bpc) + ((ri & 7) * bpc + b % bpc) * 4) >>
       (ri >= 8 ? 16 : 0)) & 0xFFFFu;
  const float d = subnormal ? ref_f16_to_f32(sbits) : __half2float(__ushort_as_half((unsigned short)sbits));
  uint32_t ot[3][16];
  for (int e = 0; e < 32; e += 2) {
    float w2[2];
    for (int u = 0; u < 2; u++) {
      const int k = b * 32 + e + u;
      int q;
      if (g.fmt == VXB_Q4_0) {
        const int step = k / 16, kk = k % 16;
        const int c = step / 4, j = step % 4;
        const int jj = kk & 3, ln = (ri & 7) * 4 + kk / 4;
        const int pos = (ri >= 8 ? 4 : 0) + (jj >= 2 ? 8 : 0) + ((jj & 1) ? 16 : 0);
        const uint32_t w = *reinterpret_cast<const uint32_t *>(tiled + tiled_codes_at(g, t, c) + ln * 16 + j * 4);
        q = (int)((w >> pos) & 0xF) - 8;
      } else {
        const int step = k / 16, kk = k % 16;
        const int c = step / 2;
        const int jj = kk & 3, ln = (ri & 7) * 4 + kk / 4;
        const int j = (step % 2) * 2 + (jj >= 2 ? 1 : 0);
        const int byte = (ri >= 8 ? 2 : 0) + (jj & 1);
        q = (int)tiled[tiled_codes_at(g, t, c) + ln * 16 + j * 4 + byte] - 128;
      }
      w2[u] = (float)q * d;
    }
    // remainders are exact in f32: each term removes the leading 8 bits
    for (int t = 0; t < 3; t++) {
      const uint32_t h = (uint32_t)f32_to_bf16_bits(w2[0]) | ((uint32_t)f32_to_bf16_bits(w2[1]) << 16);
      ot[t][e / 2] = h;
      w2[0] -= bf16_bits_to_f32(h & 0xFFFFu);
      w2[1] -= bf16_bits_to_f32(h >> 16);
    }
  }
  for (int t = 0; t < terms; t++) {
    uint4 *p = reinterpret_cast<uint4 *>(out + ((size_t)t * g.N + r) * g.K + b * 32);
    for (int i = 0; i < 4; i++) p[i] = make_uint4(ot[t][4 * i], ot[t][4 * i + 1], ot[t][4 * i + 2], ot[t][4 * i + 3]);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn(vxb_ctx *ctx) {
  static std::mutex mu;
  static EncodeTiledFn fn = nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p) {
      cudaGetLastError();
      set_error(ctx, VXB_ECUDA, "vxb_gemm_q: cuTensorMapEncodeTiled is not available from the driver");
      return nullptr;
    }
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// row-major bf16 [rows, K] -> 2-D map (k, row), box (64, box_rows), 128-byte swizzle
int make_map(vxb_ctx *ctx, EncodeTiledFn fn, CUtensorMap *map, const void *base, int rows, int K, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ctx, VXB_EINVAL, "vxb_gemm_q: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VXB_OK;
}

}  // namespace

namespace vxb {

static int gemm_terms(int fmt) { return fmt == VXB_Q4_0 ? 2 : 3; }

size_t gemm_scratch_bytes(int N, int K) { return (size_t)N * K * 2 * 3; }

int gemm_q_launch(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x, int M, int y_dtype,
                  void *d_y, const float *d_resid, void *d_scratch, cudaStream_t st) {
  if (fmt != VXB_Q4_0 && fmt != VXB_Q8_0) return set_error(ctx, VXB_EINVAL, "vxb_gemm_q: unknown format %d", fmt);
  if (N <= 0 || K <= 0 || K % 32 || M <= 0) return set_error(ctx, VXB_EINVAL, "vxb_gemm_q: bad shape M=%d N=%d K=%d", M, N, K);
  if (y_dtype != VXB_F32 && y_dtype != VXB_BF16) return set_error(ctx, VXB_EINVAL, "vxb_gemm_q: y_dtype must be F32 or BF16");
  if (!d_tiled || !d_x || !d_y || !d_scratch) return set_error(ctx, VXB_EINVAL, "vxb_gemm_q: null pointer");
  if (((uintptr_t)d_x) % 16 || ((uintptr_t)d_scratch) % 16)
    return set_error(ctx, VXB_EINVAL, "vxb_gemm_q: activations must be 16-byte aligned");
  if (int rc = ws_reserve(ctx, 0, 0)) return rc;  // device error word
  const TiledGeom g = tiled_geom(fmt, N, K);
  const int terms = gemm_terms(fmt);
  uint16_t *wt = (uint16_t *)d_scratch;
  const size_t nblk = (size_t)N * (K / 32);
  dequant_terms_kernel<<<(unsigned)((nblk + 255) / 256), 256, 0, st>>>((const uint8_t *)d_tiled, g, terms, wt);
  if (int rc = launch_check(ctx, "dequant_terms_kernel")) return rc;
  EncodeTiledFn fn = encode_fn(ctx);
  if (!fn) return VXB_ECUDA;
  CUtensorMap mx, mw;
  if (int rc = make_map(ctx, fn, &mx, d_x, M, K, BM)) return rc;
  if (int rc = make_map(ctx, fn, &mw, wt, terms * N, K, BN)) return rc;
  static std::atomic<bool> configured[64][2];  // kernel attributes set on this device (zero-initialized)
  if (!configured[ctx->device & 63][terms - 2]) {
    if (terms == 2)
      VXB_CUDA_TRY(ctx, cudaFuncSetAttribute(gemm_terms_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             GemmGeo<2>::SMEM_ALLOC));
    else
      VXB_CUDA_TRY(ctx, cudaFuncSetAttribute(gemm_terms_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             GemmGeo<3>::SMEM_ALLOC));
    configured[ctx->device & 63][terms - 2] = true;
  }
  GemmArgs a;
  a.y = d_y;
  a.resid = d_resid;
  a.err = ctx->d_err;
  a.M = M;
  a.N = N;
  a.K = K;
  a.y_dtype = y_dtype;
  // persistent CTAs, one per SM (the kernel holds an SM's shared memory)
  const long long ntile = (long long)((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int sms = ctx->num_sms > 0 ? ctx->num_sms : 148;
  dim3 grid((unsigned)std::min<long long>(ntile, sms));
  if (terms == 2)
    gemm_terms_kernel<2><<<grid, THREADS, GemmGeo<2>::SMEM_ALLOC, st>>>(mx, mw, a);
  else
    gemm_terms_kernel<3><<<grid, THREADS, GemmGeo<3>::SMEM_ALLOC, st>>>(mx, mw, a);
  return launch_check(ctx, "gemm_terms_kernel");
}

int gemm_ws_reserve(vxb_ctx *ctx, size_t bytes, void **out) {
  if (bytes > ctx->gemm_ws_bytes) {
    if (ctx->gemm_ws) {
      VXB_CUDA_TRY(ctx, cudaDeviceSynchronize());  // queued GEMMs may still read it
      VXB_CUDA_TRY(ctx, cudaFree(ctx->gemm_ws));
    }
    ctx->gemm_ws = nullptr;
    ctx->gemm_ws_bytes = 0;
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
      cudaGetLastError();
      return set_error(ctx, VXB_ENOMEM, "vxb_gemm_q: scratch of %zu bytes", bytes);
    }
    ctx->gemm_ws = p;
    ctx->gemm_ws_bytes = bytes;
  }
  *out = ctx->gemm_ws;
  return VXB_OK;
}

}  // namespace vxb

VXB_API int vxb_gemm_q(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x, int M,
                       int y_dtype, void *d_y, void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_gemm_q: null context");
  if (N <= 0 || K <= 0) return set_error(ctx, VXB_EINVAL, "vxb_gemm_q: bad shape N=%d K=%d", N, K);
  if (int rc = use_device(ctx)) return rc;
  void *scratch = nullptr;
  if (int rc = gemm_ws_reserve(ctx, gemm_scratch_bytes(N, K), &scratch)) return rc;
  return gemm_q_launch(ctx, fmt, d_tiled, N, K, d_x, M, y_dtype, d_y, nullptr, scratch, (cudaStream_t)stream);
}
