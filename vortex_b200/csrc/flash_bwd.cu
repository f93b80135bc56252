// Flash-attention backward (replaces flash_attention_backward,
// src/flash_attention.rs:227-317):
//
//   D_i  = dO_i . O_i
//   P_ij = exp(scale * q_i . k_j - lse_i)             (0 for masked keys)
//   dV_j = sum_i P_ij dO_i
//   dS_ij = P_ij (dO_i . v_j - D_i) * scale
//   dK_j = sum_i dS_ij q_i,   dQ_i = sum_j dS_ij k_j
//
// Tensors as the forward: bf16 [B, S, heads, 128] (query head h reads kv head
// h / (H / Hkv)), lse f32 [B, H, S] (natural log, the forward's second
// output); the gradients are f32, dK / dV summed over the query heads of a
// group. Three kernels, no atomics (deterministic):
//   * fb_dot_kernel: D per (b, h, i);
//   * fb_dkdv_kernel: one CTA per (64-key tile, kv head, batch) accumulates
//     dK and dV of its keys in registers over every query tile that can see
//     them (and every query head of the group);
//   * fb_dq_kernel: one CTA per (64-query tile, head, batch) accumulates dQ
//     over every key tile it can see.
// Both recompute S and dP with mma.m16n8k16 (bf16 operands, f32 accumulate);
// every operand is staged in shared memory k-contiguous (transposed copies
// where the contraction runs over queries or keys), rows padded to spread
// the banks. P and dS enter their products as bf16 hi + lo pairs (the lo
// part is the rounding residue of the hi part), so they carry ~16 bits, as
// the forward's P does.
#include <cuda_bf16.h>

#include "vxb_internal.h"

using namespace vxb;

namespace {

constexpr int FB_T = 64;       // query / key tile
constexpr int FB_D = 128;      // head dim
constexpr int FB_THREADS = 128;  // 4 warps x 16 rows
constexpr int LDD = FB_D + 8;  // row stride (elements) of [row][d] tiles
constexpr int LDT = FB_T + 8;  // row stride of [d][row] and [64][64] tiles

__device__ __forceinline__ void mma16816(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ld32(const uint16_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// hi = bf16(x), lo = bf16(x - hi)
__device__ __forceinline__ void split1(float x, uint16_t &hi, uint16_t &lo) {
  hi = f32_to_bf16_bits(x);
  lo = f32_to_bf16_bits(x - bf16_bits_to_f32(hi));
}

// C[16 rows x 8*NT cols] += A[rows r0.., k over KD] * Bt[cols.., k]^T where A
// is [row][k] (stride lda) and Bt is [col][k] (stride ldb), both bf16, for the
// warp's 16 rows; acc[nt][4] in the m16n8 C layout.
template <int NT, int KD>
__device__ __forceinline__ void warp_gemm(float (&acc)[NT][4], const uint16_t *A, int lda, int r0, const uint16_t *Bt,
                                          int ldb, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int k0 = 0; k0 < KD; k0 += 16) {
    const uint16_t *ar = A + (size_t)(r0 + g) * lda + k0 + 2 * t;
    const uint32_t a0 = ld32(ar), a1 = ld32(ar + 8 * lda), a2 = ld32(ar + 8), a3 = ld32(ar + 8 * lda + 8);
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      const uint16_t *br = Bt + (size_t)(nt * 8 + g) * ldb + k0 + 2 * t;
      mma16816(acc[nt], a0, a1, a2, a3, ld32(br), ld32(br + 8));
    }
  }
}

struct FbArgs {
  const uint16_t *q, *k, *v, *o, *dout;
  const float *lse;
  float *dq, *dk, *dv, *dvec;
  int B, H, Hkv, S;
  float scale;
  int causal;
};

__global__ void fb_dot_kernel(const FbArgs a) {
  // one warp per (b, i, h)
  const size_t w = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const size_t total = (size_t)a.B * a.S * a.H;
  if (w >= total) return;
  const int h = (int)(w % a.H);
  const size_t bi = w / a.H;
  const int i = (int)(bi % a.S), b = (int)(bi / a.S);
  const uint16_t *po = a.o + w * FB_D, *pd = a.dout + w * FB_D;
  float s = 0.f;
  for (int d = lane; d < FB_D; d += 32) s += bf16_bits_to_f32(po[d]) * bf16_bits_to_f32(pd[d]);
  s = warp_sum(s);
  if (lane == 0) a.dvec[((size_t)b * a.H + h) * a.S + i] = s;
}

// [64 rows][128] tile of a [B, S, heads, 128] tensor into smem [row][LDD]
// (rows past S zero); optionally also the transpose [128][LDT]
__device__ __forceinline__ void load_tile(const uint16_t *src, int b, int head, int heads, int S, int r0,
                                          uint16_t *dst, uint16_t *dst_t) {
  for (int c = threadIdx.x; c < FB_T * FB_D / 8; c += FB_THREADS) {
    const int r = c / (FB_D / 8), d0 = (c % (FB_D / 8)) * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r0 + r < S) v = *reinterpret_cast<const uint4 *>(src + (((size_t)b * S + r0 + r) * heads + head) * FB_D + d0);
    *reinterpret_cast<uint4 *>(dst + r * LDD + d0) = v;
    if (dst_t) {
      const uint16_t *e = reinterpret_cast<const uint16_t *>(&v);
#pragma unroll
      for (int j = 0; j < 8; j++) dst_t[(d0 + j) * LDT + r] = e[j];
    }
  }
}

// P and dS of the warp's 16 query rows x 64 keys from the S and dP fragments
// (rows qr0 + g, +8; keys kc0 + 8 nt + 2t, +1)
__device__ __forceinline__ void p_ds(const FbArgs &a, float (&s)[8][4], float (&dp)[8][4], int qr0, int kc0,
                                     const float *lse_s, const float *dv_s, int qbase, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const float L2E = 1.4426950408889634f;
#pragma unroll
  for (int nt = 0; nt < 8; nt++)
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int ql = qbase + g + (e >> 1) * 8;  // local query row in the tile
      const int qi = qr0 + ql, kj = kc0 + nt * 8 + 2 * t + (e & 1);
      const bool ok = qi < a.S && kj < a.S && !(a.causal && kj > qi);
      const float p = ok ? exp2f(s[nt][e] * a.scale * L2E - lse_s[ql] * L2E) : 0.f;
      s[nt][e] = p;
      dp[nt][e] = p * (dp[nt][e] - dv_s[ql]) * a.scale;
    }
}

__global__ void __launch_bounds__(FB_THREADS) fb_dkdv_kernel(const FbArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t *Ks = reinterpret_cast<uint16_t *>(smem);  // [key][LDD]
  uint16_t *Vs = Ks + FB_T * LDD;
  uint16_t *Qs = Vs + FB_T * LDD;                     // [q][LDD]
  uint16_t *Os = Qs + FB_T * LDD;                     // dO [q][LDD]
  uint16_t *QT = Os + FB_T * LDD;                     // [d][LDT]
  uint16_t *OT = QT + FB_D * LDT;                     // dO^T [d][LDT]
  uint16_t *PTh = OT + FB_D * LDT;                    // P^T hi [key][LDT]
  uint16_t *PTl = PTh + FB_T * LDT;
  uint16_t *STh = PTl + FB_T * LDT;                   // dS^T hi [key][LDT]
  uint16_t *STl = STh + FB_T * LDT;
  float *lse_s = reinterpret_cast<float *>(STl + FB_T * LDT);
  float *dv_s = lse_s + FB_T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int j0 = blockIdx.x * FB_T, hk = blockIdx.y, b = blockIdx.z;
  const int G = a.H / a.Hkv;
  load_tile(a.k, b, hk, a.Hkv, a.S, j0, Ks, nullptr);
  load_tile(a.v, b, hk, a.Hkv, a.S, j0, Vs, nullptr);
  float dK[16][4], dV[16][4];
#pragma unroll
  for (int n = 0; n < 16; n++)
#pragma unroll
    for (int e = 0; e < 4; e++) dK[n][e] = dV[n][e] = 0.f;
  const int i_first = a.causal ? (j0 / FB_T) * FB_T : 0;
  for (int hh = 0; hh < G; hh++) {
    const int h = hk * G + hh;
    for (int i0 = i_first; i0 < a.S; i0 += FB_T) {
      __syncthreads();  // the previous tile's operands are consumed
      load_tile(a.q, b, h, a.H, a.S, i0, Qs, QT);
      load_tile(a.dout, b, h, a.H, a.S, i0, Os, OT);
      for (int r = threadIdx.x; r < FB_T; r += FB_THREADS) {
        const bool in = i0 + r < a.S;
        lse_s[r] = in ? a.lse[((size_t)b * a.H + h) * a.S + i0 + r] : 0.f;
        dv_s[r] = in ? a.dvec[((size_t)b * a.H + h) * a.S + i0 + r] : 0.f;
      }
      __syncthreads();
      float s[8][4], dp[8][4];
#pragma unroll
      for (int n = 0; n < 8; n++)
#pragma unroll
        for (int e = 0; e < 4; e++) s[n][e] = dp[n][e] = 0.f;
      warp_gemm<8, FB_D>(s, Qs, LDD, 16 * warp, Ks, LDD, lane);
      warp_gemm<8, FB_D>(dp, Os, LDD, 16 * warp, Vs, LDD, lane);
      p_ds(a, s, dp, i0, j0, lse_s, dv_s, 16 * warp, lane);
      // P^T and dS^T (hi, lo) into [key][query]
#pragma unroll
      for (int nt = 0; nt < 8; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int ql = 16 * warp + g + (e >> 1) * 8, kl = nt * 8 + 2 * t + (e & 1);
          uint16_t hi, lo;
          split1(s[nt][e], hi, lo);
          PTh[kl * LDT + ql] = hi;
          PTl[kl * LDT + ql] = lo;
          split1(dp[nt][e], hi, lo);
          STh[kl * LDT + ql] = hi;
          STl[kl * LDT + ql] = lo;
        }
      __syncthreads();
      // dV += P^T dO, dK += dS^T Q over the tile's 64 queries (warp: 16 keys)
      warp_gemm<16, FB_T>(dV, PTh, LDT, 16 * warp, OT, LDT, lane);
      warp_gemm<16, FB_T>(dV, PTl, LDT, 16 * warp, OT, LDT, lane);
      warp_gemm<16, FB_T>(dK, STh, LDT, 16 * warp, QT, LDT, lane);
      warp_gemm<16, FB_T>(dK, STl, LDT, 16 * warp, QT, LDT, lane);
    }
  }
#pragma unroll
  for (int nt = 0; nt < 16; nt++)
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int kj = j0 + 16 * warp + g + (e >> 1) * 8, d = nt * 8 + 2 * t + (e & 1);
      if (kj < a.S) {
        const size_t o = (((size_t)b * a.S + kj) * a.Hkv + hk) * FB_D + d;
        a.dk[o] = dK[nt][e];
        a.dv[o] = dV[nt][e];
      }
    }
}

__global__ void __launch_bounds__(FB_THREADS) fb_dq_kernel(const FbArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t *Qs = reinterpret_cast<uint16_t *>(smem);  // [q][LDD]
  uint16_t *Os = Qs + FB_T * LDD;                     // dO [q][LDD]
  uint16_t *Ks = Os + FB_T * LDD;                     // [key][LDD]
  uint16_t *Vs = Ks + FB_T * LDD;
  uint16_t *KT = Vs + FB_T * LDD;                     // [d][LDT]
  float *lse_s = reinterpret_cast<float *>(KT + FB_D * LDT);
  float *dv_s = lse_s + FB_T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int i0 = blockIdx.x * FB_T, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (a.H / a.Hkv);
  load_tile(a.q, b, h, a.H, a.S, i0, Qs, nullptr);
  load_tile(a.dout, b, h, a.H, a.S, i0, Os, nullptr);
  for (int r = threadIdx.x; r < FB_T; r += FB_THREADS) {
    const bool in = i0 + r < a.S;
    lse_s[r] = in ? a.lse[((size_t)b * a.H + h) * a.S + i0 + r] : 0.f;
    dv_s[r] = in ? a.dvec[((size_t)b * a.H + h) * a.S + i0 + r] : 0.f;
  }
  float dQ[16][4];
#pragma unroll
  for (int n = 0; n < 16; n++)
#pragma unroll
    for (int e = 0; e < 4; e++) dQ[n][e] = 0.f;
  const int j_end = a.causal ? min(a.S, i0 + FB_T) : a.S;
  for (int j0 = 0; j0 < j_end; j0 += FB_T) {
    __syncthreads();
    load_tile(a.k, b, hk, a.Hkv, a.S, j0, Ks, KT);
    load_tile(a.v, b, hk, a.Hkv, a.S, j0, Vs, nullptr);
    __syncthreads();
    float s[8][4], dp[8][4];
#pragma unroll
    for (int n = 0; n < 8; n++)
#pragma unroll
      for (int e = 0; e < 4; e++) s[n][e] = dp[n][e] = 0.f;
    warp_gemm<8, FB_D>(s, Qs, LDD, 16 * warp, Ks, LDD, lane);
    warp_gemm<8, FB_D>(dp, Os, LDD, 16 * warp, Vs, LDD, lane);
    p_ds(a, s, dp, i0, j0, lse_s, dv_s, 16 * warp, lane);
    // dQ += dS K: the dS fragments of key tiles 2kk, 2kk+1 are the A fragment
    // of k-step kk (hi and lo parts); B = K^T [d][key]
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      uint32_t ah[4], al[4];
      {
        float x[8] = {dp[2 * kk][0], dp[2 * kk][1], dp[2 * kk][2], dp[2 * kk][3],
                      dp[2 * kk + 1][0], dp[2 * kk + 1][1], dp[2 * kk + 1][2], dp[2 * kk + 1][3]};
        // a0: row g keys 2t,2t+1 (tile 2kk); a1: row g+8 (tile 2kk); a2/a3: tile 2kk+1
        const int idx[4][2] = {{0, 1}, {2, 3}, {4, 5}, {6, 7}};
#pragma unroll
        for (int r = 0; r < 4; r++) {
          const float u = x[idx[r][0]], w = x[idx[r][1]];
          const uint32_t hv = pack2(u, w);
          const float uh = __uint_as_float(hv << 16), wh = __uint_as_float(hv & 0xFFFF0000u);
          ah[r] = hv;
          al[r] = pack2(u - uh, w - wh);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 16; nt++) {
        const uint16_t *br = KT + (size_t)(nt * 8 + g) * LDT + kk * 16 + 2 * t;
        const uint32_t b0 = ld32(br), b1 = ld32(br + 8);
        mma16816(dQ[nt], ah[0], ah[1], ah[2], ah[3], b0, b1);
        mma16816(dQ[nt], al[0], al[1], al[2], al[3], b0, b1);
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < 16; nt++)
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int qi = i0 + 16 * warp + g + (e >> 1) * 8, d = nt * 8 + 2 * t + (e & 1);
      if (qi < a.S) a.dq[(((size_t)b * a.S + qi) * a.H + h) * FB_D + d] = dQ[nt][e];
    }
}

}  // namespace

VXB_API int vxb_flash_bwd(vxb_ctx *ctx, const uint16_t *d_q, const uint16_t *d_k, const uint16_t *d_v,
                          const uint16_t *d_o, const uint16_t *d_dout, const float *d_lse, int B, int H, int Hkv,
                          int S, int d, float scale, int causal, float *d_dq, float *d_dk, float *d_dv, void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_flash_bwd: null context");
  if (d != FB_D) return set_error(ctx, VXB_EUNSUPPORTED, "vxb_flash_bwd: head_dim %d (128 only)", d);
  if (B <= 0 || H <= 0 || Hkv <= 0 || S <= 0 || H % Hkv)
    return set_error(ctx, VXB_EINVAL, "vxb_flash_bwd: bad shape B=%d H=%d Hkv=%d S=%d", B, H, Hkv, S);
  if (!d_q || !d_k || !d_v || !d_o || !d_dout || !d_lse || !d_dq || !d_dk || !d_dv)
    return set_error(ctx, VXB_EINVAL, "vxb_flash_bwd: null pointer");
  if (((uintptr_t)d_q | (uintptr_t)d_k | (uintptr_t)d_v) % 16)
    return set_error(ctx, VXB_EINVAL, "vxb_flash_bwd: q, k, v must be 16-byte aligned");
  if (int rc = use_device(ctx)) return rc;
  const size_t nd = (size_t)B * H * S;
  if (int rc = ws_reserve(ctx, nd * sizeof(float), 0)) return rc;
  FbArgs a;
  a.q = d_q;
  a.k = d_k;
  a.v = d_v;
  a.o = d_o;
  a.dout = d_dout;
  a.lse = d_lse;
  a.dq = d_dq;
  a.dk = d_dk;
  a.dv = d_dv;
  a.dvec = (float *)ctx->ws;
  a.B = B;
  a.H = H;
  a.Hkv = Hkv;
  a.S = S;
  a.scale = scale;
  a.causal = causal;
  cudaStream_t st = (cudaStream_t)stream;
  fb_dot_kernel<<<(unsigned)((nd + 7) / 8), 256, 0, st>>>(a);
  if (int rc = launch_check(ctx, "fb_dot_kernel")) return rc;
  const size_t sm_kv = (size_t)4 * FB_T * LDD * 2 + (size_t)2 * FB_D * LDT * 2 + (size_t)4 * FB_T * LDT * 2 + 2 * FB_T * 4;
  const size_t sm_q = (size_t)4 * FB_T * LDD * 2 + (size_t)FB_D * LDT * 2 + 2 * FB_T * 4;
  static bool configured[64];
  if (!configured[ctx->device & 63]) {
    VXB_CUDA_TRY(ctx, cudaFuncSetAttribute(fb_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_kv));
    VXB_CUDA_TRY(ctx, cudaFuncSetAttribute(fb_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_q));
    configured[ctx->device & 63] = true;
  }
  const unsigned tiles = (unsigned)((S + FB_T - 1) / FB_T);
  fb_dkdv_kernel<<<dim3(tiles, Hkv, B), FB_THREADS, sm_kv, st>>>(a);
  if (int rc = launch_check(ctx, "fb_dkdv_kernel")) return rc;
  fb_dq_kernel<<<dim3(tiles, H, B), FB_THREADS, sm_q, st>>>(a);
  return launch_check(ctx, "fb_dq_kernel");
}
