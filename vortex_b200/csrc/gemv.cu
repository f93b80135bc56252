// K1: decode dequant-GEMV / skinny GEMM over tiled Q4_0 / Q8_0 weights.
//
//   y[b, n] = sum_k deq(W)[n, k] * x[b, k]     (b < batch <= 32)
//
// Replaces weight_only_matmul (src/quantize.rs:845-852, = dequantize then
// matmul_f64 890-902) and the matmul of Linear::forward
// (src/transformer.rs:332-352) at decode batch sizes.
//
// Design (HBM-bound streaming):
//  * Each warp owns one 16-row tile and streams its 512-byte (tile, k-chunk)
//    slices with 128-bit non-allocating loads; every lane's 16 bytes are its
//    tensor-core A fragments, so codes are unpacked in registers and never
//    touch shared memory. Codes (-8..7 or -128..127) are exact in bf16:
//    Q4_0 uses the bf16 magic 128+n (1 LOP3 + 1 SUB.BF16X2 per two codes),
//    Q8_0 goes through the f32 magic 2^23+u and one CVT per two codes.
//  * The activations x (bf16) of the CTA's k-range are copied into shared
//    memory unchanged with cp.async by all threads and used directly as the
//    bf16 B operand.
//  * mma.m16n8k16 (bf16 x bf16 -> f32) forms the per-block dot products of
//    two k16 steps; the per-(row, block) f16 scale is applied in f32 to that
//    block partial, so scales never round into the operands.
//  * Split-K across CTAs with deterministic reduction: each CTA writes its
//    f32 partial to the workspace and the last CTA of a row group (counter in
//    global memory) sums the partials in split order and applies the
//    epilogue. Counters are returned to zero by that CTA.
//  * All weight loads of a warp are issued before griddepcontrol.wait, so
//    under programmatic dependent launch the weight stream of this GEMV
//    overlaps the tail of the kernel that produces x.
#include <algorithm>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gemv.h"
#include "tiled_layout.h"
#include "vxb_internal.h"

using namespace vxb;

namespace {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int ROWS_PER_CTA = WARPS * 16;

struct GemvArgs {
  const uint8_t *codes;
  const uint32_t *scales;
  const uint32_t *hdr;
  const uint16_t *x;
  void *y;
  const float *resid;  // optional residual added in the epilogue (f32 [B, N])
  float *ws;
  unsigned *counters;
  int N, K, B, n_tiles, n_chunks, n_blocks, S, y_dtype, xs_stride;
};

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t m, uint32_t o) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(m), "r"(o));
  return d;
}

__device__ __forceinline__ uint32_t bsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Q4_0 tiled word -> A fragment {a0a1, a2a3, a4a5, a6a7} of exact codes.
// Nibble n at bits 0-3 / 16-19 of (w >> 4i): bf16 0x4300|n = 128+n, minus 136.
__device__ __forceinline__ void decode_q4(uint32_t w, uint32_t A[4]) {
  const uint32_t M = 0x43004300u;    // bf16 128.0 x2
  const uint32_t SUB = 0x43084308u;  // bf16 136.0 x2
  A[0] = bsub2(lop_and_or(w, 0x000F000Fu, M), SUB);
  A[1] = bsub2(lop_and_or(w >> 4, 0x000F000Fu, M), SUB);
  A[2] = bsub2(lop_and_or(w >> 8, 0x000F000Fu, M), SUB);
  A[3] = bsub2(lop_and_or(w >> 12, 0x000F000Fu, M), SUB);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// Four int8 codes of one word -> two bf16x2 (exact): byte b -> f32 2^23 + (b^0x80)
// via PRMT, minus 2^23 + 128.
__device__ __forceinline__ void q8_word(uint32_t w, uint32_t &lo, uint32_t &hi) {
  const uint32_t u = w ^ 0x80808080u;
  const float B = 8388736.0f;  // 2^23 + 128
  const float c0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - B;
  const float c1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - B;
  const float c2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - B;
  const float c3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - B;
  lo = pack_bf16x2(c0, c1);
  hi = pack_bf16x2(c2, c3);
}

// Q8_0 tiled words (a0..a3 | a4..a7) -> A fragment of exact codes.
__device__ __forceinline__ void decode_q8(uint32_t w0, uint32_t w1, uint32_t A[4]) {
  q8_word(w0, A[0], A[1]);
  q8_word(w1, A[2], A[3]);
}

__device__ __forceinline__ void mma_bf16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1,
                                         const float c[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

__device__ __forceinline__ float2 decode_scales(uint32_t s, bool subnormal) {
  if (!subnormal) {
    __half2 h = *reinterpret_cast<__half2 *>(&s);
    return __half22float2(h);
  }
  return make_float2(ref_f16_to_f32(s & 0xFFFFu), ref_f16_to_f32(s >> 16));
}

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc, int src_bytes) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gsrc), "r"(src_bytes));
}

__device__ __forceinline__ void epilogue_store(const GemvArgs &a, int b, int row, float v) {
  const size_t o = (size_t)b * a.N + row;
  if (a.resid) v += a.resid[o];
  if (a.y_dtype == VXB_BF16)
    ((uint16_t *)a.y)[o] = f32_to_bf16_bits(v);
  else
    ((float *)a.y)[o] = v;
}

template <int FMT, int NT>
__global__ void __launch_bounds__(THREADS, 2) gemv_q_kernel(const GemvArgs a) {
  constexpr int CH = FMT == 0 ? 64 : 32;  // k per chunk
  constexpr int BPC = CH / 32;            // blocks per chunk
  constexpr int BR = 8 * NT;              // padded batch rows
  constexpr int UNROLL = NT <= 2 ? 12 : 8;  // 512-byte loads in flight per warp
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t *xs = reinterpret_cast<uint16_t *>(smem);
  float *red = reinterpret_cast<float *>(smem + (size_t)BR * a.xs_stride * 2);  // [BR][ROWS_PER_CTA]
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x, s = blockIdx.y;
  const int c0 = (int)((long long)s * a.n_chunks / a.S);
  const int c1 = (int)((long long)(s + 1) * a.n_chunks / a.S);
  const int nck = c1 - c0;
  const int k0 = c0 * CH, kc = nck * CH;
  const int tile = g * WARPS + warp;
  const bool active = tile < a.n_tiles;

  const uint4 *wp = reinterpret_cast<const uint4 *>(a.codes + ((size_t)(active ? tile : 0) * a.n_chunks + c0) * 512) + lane;
  const uint32_t *sp = a.scales + ((size_t)(active ? tile : 0) * a.n_blocks + (size_t)c0 * BPC) * 8 + (lane >> 2);

  // Issue the first batch of weight loads before waiting on the producer of x.
  uint4 wv[UNROLL];
  uint32_t sv[UNROLL][BPC];
#pragma unroll
  for (int u = 0; u < UNROLL; u++) {
    if (active && u < nck) {
      wv[u] = ldg_stream(wp + (size_t)u * 32);
#pragma unroll
      for (int bb = 0; bb < BPC; bb++) sv[u][bb] = __ldg(sp + ((size_t)u * BPC + bb) * 8);
    }
  }
  const bool subnormal = (__ldg(a.hdr + 1) & TILED_FLAG_SUBNORMAL_SCALES) != 0;

  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // Stage x[:, k0:k0+kc] (bf16, unchanged) with 16-byte async copies; rows
  // past the batch and columns past K are zero-filled.
  {
    const int per_row = kc / 8;  // 16-byte pieces per row
    const int total = BR * per_row;
    for (int i = threadIdx.x; i < total; i += THREADS) {
      const int b = i / per_row, p = i % per_row;
      const int kk = k0 + p * 8;
      const bool ok = b < a.B && kk < a.K;
      const uint16_t *src = ok ? a.x + (size_t)b * a.K + kk : a.x;
      cp_async16(xs + (size_t)b * a.xs_stride + p * 8, src, ok ? 16 : 0);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  }
  __syncthreads();

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[nt][i] = 0.f;

  if (active) {
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
    const int q2 = (lane & 3) * 2;
    const uint16_t *xrow = xs + (size_t)(lane >> 2) * a.xs_stride + q2;
    // Rolling pipeline: slot u holds chunk ci+u; after taking it, the slot is
    // refilled with chunk ci+u+UNROLL so UNROLL loads stay in flight.
    for (int ci = 0; ci < nck; ci += UNROLL) {
#pragma unroll
      for (int u = 0; u < UNROLL; u++) {
        if (ci + u < nck) {
          const uint4 cur = wv[u];
          uint32_t cs[BPC];
#pragma unroll
          for (int bb = 0; bb < BPC; bb++) cs[bb] = sv[u][bb];
          const int nxt = ci + u + UNROLL;
          if (nxt < nck) {
            wv[u] = ldg_stream(wp + (size_t)nxt * 32);
#pragma unroll
            for (int bb = 0; bb < BPC; bb++) sv[u][bb] = __ldg(sp + ((size_t)nxt * BPC + bb) * 8);
          }
          const uint32_t *wu = reinterpret_cast<const uint32_t *>(&cur);
#pragma unroll
          for (int bb = 0; bb < BPC; bb++) {
            float t[NT][4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
              uint32_t A[4];
              if (FMT == 0)
                decode_q4(wu[bb * 2 + h], A);
              else
                decode_q8(wu[h * 2], wu[h * 2 + 1], A);
              const int kk = (ci + u) * CH + (bb * 2 + h) * 16;
#pragma unroll
              for (int nt = 0; nt < NT; nt++) {
                const uint16_t *xp = xrow + (size_t)nt * 8 * a.xs_stride + kk;
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(xp);
                const uint32_t b1 = *reinterpret_cast<const uint32_t *>(xp + 8);
                mma_bf16(t[nt], A, b0, b1, h == 0 ? zero : t[nt]);
              }
            }
            const float2 d = decode_scales(cs[bb], subnormal);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
              acc[nt][0] = fmaf(d.x, t[nt][0], acc[nt][0]);
              acc[nt][1] = fmaf(d.x, t[nt][1], acc[nt][1]);
              acc[nt][2] = fmaf(d.y, t[nt][2], acc[nt][2]);
              acc[nt][3] = fmaf(d.y, t[nt][3], acc[nt][3]);
            }
          }
        }
      }
    }
  }

  // Fragments -> red[b][row].
  {
    const int rl = warp * 16 + (lane >> 2);
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      const int b = nt * 8 + (lane & 3) * 2;
      red[(size_t)b * ROWS_PER_CTA + rl] = acc[nt][0];
      red[(size_t)(b + 1) * ROWS_PER_CTA + rl] = acc[nt][1];
      red[(size_t)b * ROWS_PER_CTA + rl + 8] = acc[nt][2];
      red[(size_t)(b + 1) * ROWS_PER_CTA + rl + 8] = acc[nt][3];
    }
  }
  __syncthreads();

  const int row0 = g * ROWS_PER_CTA;
  const int nrows = min(ROWS_PER_CTA, a.N - row0);
  const int nel = a.B * ROWS_PER_CTA;
  if (a.S == 1) {
    for (int i = threadIdx.x; i < nel; i += THREADS) {
      const int b = i / ROWS_PER_CTA, r = i % ROWS_PER_CTA;
      if (r < nrows) epilogue_store(a, b, row0 + r, red[i]);
    }
    return;
  }
  const size_t NP = (size_t)a.n_tiles * 16;
  for (int i = threadIdx.x; i < nel; i += THREADS) {
    const int b = i / ROWS_PER_CTA, r = i % ROWS_PER_CTA;
    if (r < nrows) __stcg(a.ws + ((size_t)s * a.B + b) * NP + row0 + r, red[i]);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(a.counters + g, 1u);
    s_last = prev == (unsigned)(a.S - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < nel; i += THREADS) {
    const int b = i / ROWS_PER_CTA, r = i % ROWS_PER_CTA;
    if (r >= nrows) continue;
    float v = 0.f;
    for (int ss = 0; ss < a.S; ss++) v += __ldcg(a.ws + ((size_t)ss * a.B + b) * NP + row0 + r);
    epilogue_store(a, b, row0 + r, v);
  }
  if (threadIdx.x == 0) a.counters[g] = 0u;
}

template <int FMT, int NT>
int launch_t(vxb_ctx *ctx, const GemvArgs &a, dim3 grid, size_t smem, cudaStream_t st, bool pdl) {
  auto kfn = gemv_q_kernel<FMT, NT>;
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
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  VXB_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kfn, a));
  return VXB_OK;
}

}  // namespace

namespace vxb {

size_t gemv_smem_bytes(int fmt, int N, int K, int batch, int S) {
  const TiledGeom g = tiled_geom(fmt, N, K);
  const int NT = (batch + 7) / 8;
  const int kc_max = (g.n_chunks + S - 1) / S * g.chunk;
  return (size_t)8 * NT * (kc_max + 8) * 2 + (size_t)8 * NT * ROWS_PER_CTA * 4;
}

GemvPlan gemv_plan(const vxb_ctx *ctx, int fmt, int N, int K, int batch) {
  const TiledGeom g = tiled_geom(fmt, N, K);
  const int row_groups = (g.n_tiles + WARPS - 1) / WARPS;
  const int sms = ctx->num_sms > 0 ? ctx->num_sms : 148;
  const int slots = 2 * sms;  // resident CTAs (register-limited to two per SM)
  // Each CTA streams at a latency-bound rate, so the run time is the number of
  // CTA waves times the duration of one CTA (proportional to 1/S): pick the
  // split count that minimises waves/S, with a small cost per extra wave.
  int best = 1;
  double best_cost = 1e30;
  const int smax = std::min(16, std::max(1, g.n_chunks / 2));
  for (int S = 1; S <= smax; S++) {
    if (gemv_smem_bytes(fmt, N, K, batch, S) > 96 * 1024) continue;
    const int waves = (row_groups * S + slots - 1) / slots;
    const double cost = (double)waves / S + 0.03 * waves;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = S;
    }
  }
  int S = best;
  while (S < g.n_chunks && gemv_smem_bytes(fmt, N, K, batch, S) > 96 * 1024) S++;
  GemvPlan p;
  p.S = S;
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
  const TiledGeom g = tiled_geom(fmt, N, K);
  GemvPlan p = plan_override ? *plan_override : gemv_plan(ctx, fmt, N, K, batch);
  const int NT = (batch + 7) / 8;
  const int row_groups = (g.n_tiles + WARPS - 1) / WARPS;
  if (p.S > 1) {
    if (int rc = ws_reserve(ctx, (size_t)p.S * batch * g.N_pad * sizeof(float), (size_t)row_groups)) return rc;
  }
  GemvArgs a;
  const uint8_t *base = (const uint8_t *)d_tiled;
  a.codes = base + g.codes_off;
  a.scales = (const uint32_t *)(base + g.codes_off + g.codes_bytes);
  a.hdr = (const uint32_t *)base;
  a.x = d_x;
  a.y = d_y;
  a.resid = d_resid;
  a.ws = (float *)ctx->ws;
  a.counters = ctx->counters;
  a.N = N;
  a.K = K;
  a.B = batch;
  a.n_tiles = g.n_tiles;
  a.n_chunks = g.n_chunks;
  a.n_blocks = g.n_blocks;
  a.S = p.S;
  a.y_dtype = y_dtype;
  const int kc_max = (g.n_chunks + p.S - 1) / p.S * g.chunk;
  a.xs_stride = kc_max + 8;
  const size_t smem = gemv_smem_bytes(fmt, N, K, batch, p.S);
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
