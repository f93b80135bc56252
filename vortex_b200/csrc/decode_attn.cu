// K4: split-K decode attention over the paged KV cache.
//
// Replaces paged_attention / kv_cache_attention (src/kv_cache.rs:95-112,
// 207-218): for one new query per sequence,
//   out[h] = softmax(q_h . K^T * scale) V      (all cached tokens, no mask)
// generalised to [num_q_heads, head_dim] queries with grouped-query sharing
// (q head j reads kv head j / (Hq/Hkv)); Hq == Hkv == 1 is the reference case.
//
// One CTA = (sequence, kv head, token split); its four warps stream 16-token
// pages of K and V from the pool into XOR-swizzled shared memory with
// double-buffered cp.async, and compute on tensor cores:
//   S = Q K^T   : mma.m16n8k16 bf16, A = the G query heads of the group
//                 (rows padded to 16), B = K rows via ldmatrix
//   online softmax on the S fragments (exp2, per-row max/sum kept in f32,
//                 quad shuffles for the row reductions)
//   O += P V    : A = P re-packed from the S fragments, B = V via ldmatrix.trans
// Warps merge through shared memory; splits merge deterministically in the
// last-arriving CTA of each (sequence, kv head) (counter in global memory).
// int8 caches stage the raw int8 pages (16-byte chunks XOR-swizzled) and one
// f32 scale per (token, head), and build the MMA fragments straight from
// them: ldmatrix gives each lane 4 bytes of one K row (with the head
// dimension permuted the same way in q) or, with .trans, 2 tokens x 2
// columns of V; XOR 0x80, a byte permute with the f16 magic 0x64 and one
// f16 subtraction turn two codes into exact f16 integers. q is f16 scaled
// per row by 2^-e (exact for every element within 2^-28 of the row maximum),
// P times the V scale is split into f16 hi + lo scaled by 2^k, k chosen per
// page from the page's largest V scale (O is rescaled with the softmax
// correction when k drops). The K scale multiplies the scores.
#include <atomic>
#include <climits>
#include <cstdlib>
#include <cuda_bf16.h>

#include "decode_attn.h"
#include "kv_cache.h"

using namespace vxb;

namespace {

constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int PAGE = 16;
constexpr int kMaxInlineRows = 256;

struct DecodeArgs {
  const uint16_t *q;  // [n, Hq, D] bf16
  uint16_t *out;      // [n, Hq, D] bf16
  float *lse;         // optional [n, Hq] natural-log sum-exp
  const void *pool_k, *pool_v;
  const float *sk, *sv;
  const int32_t *tables;  // this layer: [max_seqs][mbps]
  const int32_t *lens;    // this layer: [max_seqs]
  const int32_t *slots;   // [n] in device memory, or null: use slots_inline
  float *ws_o, *ws_ml;
  unsigned *counters;
  int n, Hq, Hkv, G, bs, mbps, splits, tps;
  float scale_log2;
  // slot ids passed by value (kernel parameters are captured with a graph
  // node, so a standalone call stays valid under stream capture)
  int32_t slots_inline[kMaxInlineRows];
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes));
}

// 16-byte copy at compile-time offsets from a shared and a global base
template <int SOFF, int GOFF>
__device__ __forceinline__ void cp_async16_at(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0+%2], [%1+%3], 16;" ::"r"(dst), "l"(src), "n"(SOFF), "n"(GOFF));
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src, int bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(bytes));
}

__device__ __forceinline__ void mma_bf16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// (a, b) -> hi = bf16x2(a, b) and lo = bf16x2(a - hi.a, b - hi.b)
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t &hi, uint32_t &lo) {
  hi = pack_bf16x2(a, b);
  const float ha = __uint_as_float(hi << 16), hb = __uint_as_float(hi & 0xFFFF0000u);
  lo = pack_bf16x2(a - ha, b - hb);
}

__device__ __forceinline__ void mma_f16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ __forceinline__ float2 f16x2_to_f32(uint32_t v) {
  return __half22float2(*reinterpret_cast<const __half2 *>(&v));
}

// (a, b) -> hi = f16x2(a, b) and lo = f16x2(a - hi.a, b - hi.b)
__device__ __forceinline__ void split_f16x2(float a, float b, uint32_t &hi, uint32_t &lo) {
  hi = pack_f16x2(a, b);
  const float2 h = f16x2_to_f32(hi);
  lo = pack_f16x2(a - h.x, b - h.y);
}

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Two int8 codes of w (bytes selected by `sel` with the magic byte 0x64 in
// the high halves) -> f16x2 of the exact codes: (b ^ 0x80) = c + 128 in the
// low byte of f16 0x64xx is 1024 + c + 128, minus 1152.
__device__ __forceinline__ uint32_t i8pair_f16(uint32_t w_xor80, uint32_t sel) {
  return hsub2_u(__byte_perm(w_xor80, 0x64646464u, sel), 0x64806480u);
}

// 2^x, the special-function unit's approximation (flushes results below
// 2^-126 to zero; -inf gives 0)
__device__ __forceinline__ float ex2a(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// v * 2^e for |e| <= 252 (two exact power-of-two factors)
__device__ __forceinline__ float mul_pow2f(float v, int e) {
  const int e1 = e / 2, e2 = e - e1;
  return v * __int_as_float((127 + e1) << 23) * __int_as_float((127 + e2) << 23);
}

// byte offset of 16-byte chunk c of token row r in a raw int8 page: the
// chunks of 8 consecutive rows land in distinct bank groups for ldmatrix
template <int D>
__device__ __forceinline__ uint32_t swz_raw(int r, int c) {
  if (D == 128) return (uint32_t)(r * D + ((c ^ (r & 7)) << 4));
  return (uint32_t)(r * D + ((c ^ ((r >> 1) & 3)) << 4));
}

// byte offset of 16-byte chunk c of token row r in a swizzled page tile
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * D * 2 + ((c ^ (r & 7)) << 4));
}

template <int D, bool INT8>
struct Smem {
  // per warp, per stage: bf16 tiles, or raw int8 pages and their scales
  static constexpr int TILE = PAGE * D * 2;                  // one bf16 page tile
  static constexpr int RAW = INT8 ? PAGE * D : 0;            // one int8 page
  static constexpr int SC = INT8 ? PAGE * 4 : 0;             // per-token scales
  static constexpr int STAGE = INT8 ? 2 * RAW + 2 * SC : 2 * TILE;
  static constexpr int WARP = 2 * STAGE;
  static constexpr int TOTAL = WARPS * WARP;
};

template <int D, bool INT8>
__global__ void __launch_bounds__(THREADS) decode_attn_kernel(const DecodeArgs a) {
  using SM = Smem<D, INT8>;
  constexpr int CHUNKS = D / 8;  // 16-byte chunks per bf16 row
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q4 = lane & 3;
  const int i = blockIdx.x / a.Hkv, h = blockIdx.x % a.Hkv, split = blockIdx.y;
  // programmatic dependent launch: the next kernel may launch (and prefetch
  // its weights) now; q, the lengths, block tables and pages come from earlier
  // kernels and are read after the wait through L2 only (cp.async.cg,
  // ld.global.cg): a kernel launched ahead can share an SM with an earlier
  // kernel whose L1 lines predate the data
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int slot = a.slots ? __ldcg(a.slots + i) : a.slots_inline[i];
  const int len = slot >= 0 ? __ldcg(a.lens + slot) : 0;
  const int t0 = split * a.tps;
  const int t1 = min(len, t0 + a.tps);
  const int32_t *table = a.tables + (size_t)(slot >= 0 ? slot : 0) * a.mbps;
  uint8_t *wsm = smem + (size_t)warp * SM::WARP;
  const uint32_t wsm_s = (uint32_t)__cvta_generic_to_shared(wsm);

  // Q fragments (rows = the G query heads of this group, padded to 16);
  // rs0 / rs1 multiply the scores of rows g / g+8
  uint32_t qa[D / 16][4];
  float rs0 = a.scale_log2, rs1 = a.scale_log2;
  if constexpr (INT8) {
    // f16 * 2^-e per row (max |q| * 2^-e in [2^14, 2^15)), head dimension
    // permuted like the K fragments: lane quad q4 of k16 step ks holds
    // d = 16 ks + 4 q4 .. +3 (fragment columns 2q4, 2q4+1, 2q4+8, 2q4+9)
    const uint2 *qrow0 = reinterpret_cast<const uint2 *>(a.q + ((size_t)i * a.Hq + (size_t)h * a.G + g) * D);
    const uint2 *qrow1 = reinterpret_cast<const uint2 *>(a.q + ((size_t)i * a.Hq + (size_t)h * a.G + g + 8) * D);
    const bool v0 = g < a.G, v1 = g + 8 < a.G;
    uint2 r0[D / 16], r1[D / 16];
    unsigned mx0 = 0, mx1 = 0;
#pragma unroll
    for (int ks = 0; ks < D / 16; ks++) {
      r0[ks] = v0 ? __ldcg(qrow0 + ks * 4 + q4) : make_uint2(0u, 0u);
      r1[ks] = v1 ? __ldcg(qrow1 + ks * 4 + q4) : make_uint2(0u, 0u);
      mx0 = max(mx0, max(max(r0[ks].x & 0x7FFFu, (r0[ks].x >> 16) & 0x7FFFu), max(r0[ks].y & 0x7FFFu, (r0[ks].y >> 16) & 0x7FFFu)));
      mx1 = max(mx1, max(max(r1[ks].x & 0x7FFFu, (r1[ks].x >> 16) & 0x7FFFu), max(r1[ks].y & 0x7FFFu, (r1[ks].y >> 16) & 0x7FFFu)));
    }
    mx0 = max(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = max(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = max(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = max(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const int e0 = (mx0 != 0 && mx0 < 0x7F80u) ? max((int)(mx0 >> 7), 1) - 127 - 14 : 0;
    const int e1 = (mx1 != 0 && mx1 < 0x7F80u) ? max((int)(mx1 >> 7), 1) - 127 - 14 : 0;
    auto cvt = [](uint32_t w, int e) {
      return pack_f16x2(mul_pow2f(__uint_as_float(w << 16), -e), mul_pow2f(__uint_as_float(w & 0xFFFF0000u), -e));
    };
#pragma unroll
    for (int ks = 0; ks < D / 16; ks++) {
      qa[ks][0] = cvt(r0[ks].x, e0);
      qa[ks][1] = cvt(r1[ks].x, e1);
      qa[ks][2] = cvt(r0[ks].y, e0);
      qa[ks][3] = cvt(r1[ks].y, e1);
    }
    rs0 = mul_pow2f(a.scale_log2, e0);
    rs1 = mul_pow2f(a.scale_log2, e1);
  } else {
    const uint32_t *qrow0 = reinterpret_cast<const uint32_t *>(a.q + ((size_t)i * a.Hq + (size_t)h * a.G + g) * D);
    const uint32_t *qrow1 = reinterpret_cast<const uint32_t *>(a.q + ((size_t)i * a.Hq + (size_t)h * a.G + g + 8) * D);
    const bool v0 = g < a.G, v1 = g + 8 < a.G;
#pragma unroll
    for (int ks = 0; ks < D / 16; ks++) {
      qa[ks][0] = v0 ? __ldcg(qrow0 + ks * 8 + q4) : 0u;
      qa[ks][1] = v1 ? __ldcg(qrow1 + ks * 8 + q4) : 0u;
      qa[ks][2] = v0 ? __ldcg(qrow0 + ks * 8 + 4 + q4) : 0u;
      qa[ks][3] = v1 ? __ldcg(qrow1 + ks * 8 + 4 + q4) : 0u;
    }
  }

  float o[D / 8][4];
#pragma unroll
  for (int dt = 0; dt < D / 8; dt++) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  int kcur = INT_MAX;  // int8: O is in units of 2^-kcur (P scaled by 2^kcur); INT_MAX: not set yet

  const int pg0 = t0 / PAGE, pg1 = t1 > t0 ? (t1 + PAGE - 1) / PAGE : pg0;
  const int npages = pg1 - pg0;
  const int my = npages > warp ? (npages - warp + WARPS - 1) / WARPS : 0;

  // d = 128, whole pages: lane L copies, for i = 0..7, physical 16-byte chunk
  // L % 16 of token row 2i + L / 16, i.e. the logical chunk that the swizzle
  // puts there; the shared offsets step by 512 bytes, the global ones repeat
  // every four rows, so each copy is a base register plus an immediate
  const int cr0 = lane >> 4, cpc = lane & 15;
  const uint32_t c_soff = (uint32_t)(cr0 * 256 + cpc * 16);
  int c_goff[4];
#pragma unroll
  for (int k = 0; k < 4; k++) c_goff[k] = cr0 * 256 + ((cpc ^ ((2 * k + cr0) & 7)) << 4) + k * 512;
  auto prefetch = [&](int j, int stage) {
    const int p = pg0 + warp + j * WARPS;
    const int tok0 = p * PAGE;
    // blocks of one page (the usual 16 tokens) need no division
    const int block = __ldcg(table + (a.bs == PAGE ? p : tok0 / a.bs));
    const int off = a.bs == PAGE ? 0 : tok0 % a.bs;
    const size_t base = ((size_t)block * a.Hkv + h) * a.bs + off;  // token row index in pool
    uint8_t *st = wsm + stage * SM::STAGE;
    const uint32_t st_s = wsm_s + stage * SM::STAGE;
    if (!INT8) {
      const uint16_t *kp = reinterpret_cast<const uint16_t *>(a.pool_k) + base * D;
      const uint16_t *vp = reinterpret_cast<const uint16_t *>(a.pool_v) + base * D;
      if (D == 128 && tok0 + PAGE <= len) {
        const char *kb = reinterpret_cast<const char *>(kp), *vb = reinterpret_cast<const char *>(vp);
        const char *k0 = kb + c_goff[0], *k1 = kb + c_goff[1], *k2 = kb + c_goff[2], *k3 = kb + c_goff[3];
        const char *v0 = vb + c_goff[0], *v1 = vb + c_goff[1], *v2 = vb + c_goff[2], *v3 = vb + c_goff[3];
        const uint32_t ks = st_s + c_soff, vs = st_s + SM::TILE + c_soff;
        cp_async16_at<0 * 512, 0>(ks, k0);
        cp_async16_at<1 * 512, 0>(ks, k1);
        cp_async16_at<2 * 512, 0>(ks, k2);
        cp_async16_at<3 * 512, 0>(ks, k3);
        cp_async16_at<4 * 512, 2048>(ks, k0);
        cp_async16_at<5 * 512, 2048>(ks, k1);
        cp_async16_at<6 * 512, 2048>(ks, k2);
        cp_async16_at<7 * 512, 2048>(ks, k3);
        cp_async16_at<0 * 512, 0>(vs, v0);
        cp_async16_at<1 * 512, 0>(vs, v1);
        cp_async16_at<2 * 512, 0>(vs, v2);
        cp_async16_at<3 * 512, 0>(vs, v3);
        cp_async16_at<4 * 512, 2048>(vs, v0);
        cp_async16_at<5 * 512, 2048>(vs, v1);
        cp_async16_at<6 * 512, 2048>(vs, v2);
        cp_async16_at<7 * 512, 2048>(vs, v3);
      } else if (tok0 + PAGE <= len) {
#pragma unroll
        for (int c = lane; c < PAGE * CHUNKS; c += 32) {
          const int r = c / CHUNKS, cc = c % CHUNKS;
          cp_async16(st_s + swz<D>(r, cc), kp + (size_t)r * D + cc * 8, 16);
          cp_async16(st_s + SM::TILE + swz<D>(r, cc), vp + (size_t)r * D + cc * 8, 16);
        }
      } else {
#pragma unroll
        for (int c = lane; c < PAGE * CHUNKS; c += 32) {
          const int r = c / CHUNKS, cc = c % CHUNKS;
          const int bytes = tok0 + r < len ? 16 : 0;
          cp_async16(st_s + swz<D>(r, cc), kp + (size_t)r * D + cc * 8, bytes);
          cp_async16(st_s + SM::TILE + swz<D>(r, cc), vp + (size_t)r * D + cc * 8, bytes);
        }
      }
    } else {
      const int8_t *kp = reinterpret_cast<const int8_t *>(a.pool_k) + base * D;
      const int8_t *vp = reinterpret_cast<const int8_t *>(a.pool_v) + base * D;
      constexpr int RCH = D / 16;  // 16-byte chunks per int8 row
#pragma unroll
      for (int c = lane; c < PAGE * RCH; c += 32) {
        const int r = c / RCH, cc = c % RCH;
        const int bytes = tok0 + r < len ? 16 : 0;
        cp_async16(st_s + swz_raw<D>(r, cc), kp + (size_t)r * D + cc * 16, bytes);
        cp_async16(st_s + SM::RAW + swz_raw<D>(r, cc), vp + (size_t)r * D + cc * 16, bytes);
      }
      {
        // per-token scales: lanes 0-15 the K scales, lanes 16-31 the V scales
        // (4-byte copies exist only in the L1-allocating form; a token's scale
        // is written once, by its append, before any attention reads it)
        const bool isv = lane >= 16;
        const int r = lane & 15;
        cp_async4(st_s + 2 * SM::RAW + (isv ? SM::SC : 0) + r * 4, (isv ? a.sv : a.sk) + base + r,
                  tok0 + r < len ? 4 : 0);
      }
      (void)st;
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  if (my > 0) prefetch(0, 0);
  for (int j = 0; j < my; j++) {
    const int stage = j & 1;
    if (j + 1 < my) {
      prefetch(j + 1, stage ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncwarp();
    const int p = pg0 + warp + j * WARPS;
    const int tok0 = p * PAGE;
    uint32_t kt = wsm_s + stage * SM::STAGE, vt = kt + SM::TILE;
    float ksc[2][2], vsc[2][2];
    float kfac = 1.f;  // O correction when this page lowers kcur
    if (INT8) {
      // scales of this lane's token columns (tok 2q, 2q+1 of each n-tile)
      const float *scs = reinterpret_cast<const float *>(wsm + stage * SM::STAGE + 2 * SM::RAW);
#pragma unroll
      for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const int r = nt * 8 + q4 * 2 + e;
          const bool ok = tok0 + r < len;
          ksc[nt][e] = ok ? scs[r] : 0.f;
          vsc[nt][e] = ok ? scs[PAGE + r] : 0.f;
        }
      // this page's P scaling 2^kp from its largest V scale (P * scale < 2^15)
      float vm = fmaxf(fmaxf(vsc[0][0], vsc[0][1]), fmaxf(vsc[1][0], vsc[1][1]));
      const unsigned vmb = __reduce_max_sync(0xffffffffu, __float_as_uint(vm));
      if (vmb != 0u) {
        const int kp = min(120, max(-120, 14 - ((int)((vmb >> 23) & 0xFFu) - 127)));
        if (kp < kcur) {
          kfac = kcur == INT_MAX ? 1.f : (kp - kcur >= -126 ? __int_as_float((127 + kp - kcur) << 23) : 0.f);
          kcur = kp;
        }
      }
    }
    // S = Q K^T for the page's 16 tokens (two n-tiles of 8)
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    if constexpr (INT8) {
      // ldmatrix on the raw page: matrix mi = tokens 8 (mi & 1) .. +7 of
      // 16-byte chunk 2 ks2 + (mi >> 1); lane (g, q4) gets bytes 4 q4 .. +3
      // of token g, the fragment columns {2q4, 2q4+1 | 2q4+8, 2q4+9}
      const uint32_t kr = wsm_s + stage * SM::STAGE;
      const int mi = lane >> 3;
      const int tok = (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int ks2 = 0; ks2 < D / 32; ks2++) {
        uint32_t w[4];
        ldsm_x4(kr + swz_raw<D>(tok, 2 * ks2 + (mi >> 1)), w[0], w[1], w[2], w[3]);
#pragma unroll
        for (int m = 0; m < 4; m++) {
          const uint32_t u = w[m] ^ 0x80808080u;
          mma_f16(s[m & 1], qa[2 * ks2 + (m >> 1)], i8pair_f16(u, 0x4140), i8pair_f16(u, 0x4342));
        }
      }
    } else {
#pragma unroll
      for (int ks = 0; ks < D / 16; ks++) {
        const int r = (lane >> 4) * 8 + (lane & 7);
        const int c = ks * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kt + swz<D>(r, c), b0, b1, b2, b3);
        mma_bf16(s[0], qa[ks], b0, b1);
        mma_bf16(s[1], qa[ks], b2, b3);
      }
    }
    // scale, mask (pages inside the sequence need none), online softmax.
    // bf16 with a positive scale: the scale enters the exponent's FMA (the
    // row maximum of s * rs is rs times the maximum of s)
    const bool full = tok0 + PAGE <= len;
    const bool fold = !INT8 && rs0 > 0.f && rs1 > 0.f;
    if (!fold) {
#pragma unroll
      for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          float v = s[nt][e] * (e < 2 ? rs0 : rs1);
          if (INT8) v *= ksc[nt][e & 1];
          s[nt][e] = v;
        }
    }
    if (!full) {
#pragma unroll
      for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (tok0 + nt * 8 + q4 * 2 + (e & 1) >= len) s[nt][e] = -INFINITY;
    }
    float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    if (fold) {
      mx0 *= rs0;
      mx1 *= rs1;
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = mn0 == -INFINITY ? 1.f : ex2a(m0 - mn0);
    const float c1 = mn1 == -INFINITY ? 1.f : ex2a(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float pp[2][4];
    const float f0 = fold ? rs0 : 1.f, f1 = fold ? rs1 : 1.f;
    if (__all_sync(0xffffffffu, mn0 != -INFINITY && mn1 != -INFINITY)) {
#pragma unroll
      for (int nt = 0; nt < 2; nt++) {
        pp[nt][0] = ex2a(fmaf(s[nt][0], f0, -mn0));
        pp[nt][1] = ex2a(fmaf(s[nt][1], f0, -mn0));
        pp[nt][2] = ex2a(fmaf(s[nt][2], f1, -mn1));
        pp[nt][3] = ex2a(fmaf(s[nt][3], f1, -mn1));
      }
    } else {
      // rows with no visible token yet (max -inf) get P = 0
#pragma unroll
      for (int nt = 0; nt < 2; nt++) {
        pp[nt][0] = mn0 == -INFINITY ? 0.f : ex2a(fmaf(s[nt][0], f0, -mn0));
        pp[nt][1] = mn0 == -INFINITY ? 0.f : ex2a(fmaf(s[nt][1], f0, -mn0));
        pp[nt][2] = mn1 == -INFINITY ? 0.f : ex2a(fmaf(s[nt][2], f1, -mn1));
        pp[nt][3] = mn1 == -INFINITY ? 0.f : ex2a(fmaf(s[nt][3], f1, -mn1));
      }
    }
    l0 = l0 * c0 + (pp[0][0] + pp[0][1] + pp[1][0] + pp[1][1]);
    l1 = l1 * c1 + (pp[0][2] + pp[0][3] + pp[1][2] + pp[1][3]);
    // O's correction (int8: times 2^(kp - k) when this page lowered k),
    // skipped by the whole warp when no row's maximum moved (most pages after
    // the first few: the factor is exactly 1)
    const float oc0 = c0 * kfac, oc1 = c1 * kfac;
    if (__any_sync(0xffffffffu, oc0 != 1.f || oc1 != 1.f)) {
#pragma unroll
      for (int dt = 0; dt < D / 8; dt++) {
        o[dt][0] *= oc0;
        o[dt][1] *= oc0;
        o[dt][2] *= oc1;
        o[dt][3] *= oc1;
      }
    }
    uint32_t pa[4], pl[4];
    if constexpr (INT8) {
      // P * V scale * 2^k as f16 hi + lo (22 significant bits)
      const float k2 = kcur == INT_MAX ? 1.f : mul_pow2f(1.f, kcur);
#pragma unroll
      for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) pp[nt][e] *= vsc[nt][e & 1] * k2;
      split_f16x2(pp[0][0], pp[0][1], pa[0], pl[0]);
      split_f16x2(pp[0][2], pp[0][3], pa[1], pl[1]);
      split_f16x2(pp[1][0], pp[1][1], pa[2], pl[2]);
      split_f16x2(pp[1][2], pp[1][3], pa[3], pl[3]);
      // ldmatrix.trans on the raw V page: lane (g, q4) gets V[2q4][2g],
      // V[2q4][2g+1], V[2q4+1][2g], V[2q4+1][2g+1] of its 8-token x 16-byte
      // matrix; bytes (0, 2) are the B fragment of column 2g (the even
      // n-tile of the chunk), bytes (1, 3) of column 2g + 1 (the odd one)
      const uint32_t vr = wsm_s + stage * SM::STAGE + SM::RAW;
      const int mi = lane >> 3;
      const int tok = (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int cc2 = 0; cc2 < D / 32; cc2++) {
        uint32_t w[4];
        ldsm_x4_t(vr + swz_raw<D>(tok, 2 * cc2 + (mi >> 1)), w[0], w[1], w[2], w[3]);
#pragma unroll
        for (int cp = 0; cp < 2; cp++) {
          const uint32_t ua = w[2 * cp] ^ 0x80808080u, ub = w[2 * cp + 1] ^ 0x80808080u;
          const int nt = 2 * (2 * cc2 + cp);
          const uint32_t e0 = i8pair_f16(ua, 0x4240), e1 = i8pair_f16(ub, 0x4240);
          const uint32_t d0 = i8pair_f16(ua, 0x4341), d1 = i8pair_f16(ub, 0x4341);
          mma_f16(o[nt], pa, e0, e1);
          mma_f16(o[nt], pl, e0, e1);
          mma_f16(o[nt + 1], pa, d0, d1);
          mma_f16(o[nt + 1], pl, d0, d1);
        }
      }
    } else {
    // P = P_hi + P_lo, both bf16 (P_lo = the rounding residue of P_hi), so
    // the two PV products carry P to ~2^-17 relative.
    split_bf16x2(pp[0][0], pp[0][1], pa[0], pl[0]);
    split_bf16x2(pp[0][2], pp[0][3], pa[1], pl[1]);
    split_bf16x2(pp[1][0], pp[1][1], pa[2], pl[2]);
    split_bf16x2(pp[1][2], pp[1][3], pa[3], pl[3]);
#pragma unroll
    for (int dt2 = 0; dt2 < D / 16; dt2++) {
      const int r = ((lane >> 3) & 1) * 8 + (lane & 7);
      const int c = dt2 * 2 + (lane >> 4);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vt + swz<D>(r, c), b0, b1, b2, b3);
      mma_bf16(o[2 * dt2], pa, b0, b1);
      mma_bf16(o[2 * dt2 + 1], pa, b2, b3);
      mma_bf16(o[2 * dt2], pl, b0, b1);
      mma_bf16(o[2 * dt2 + 1], pl, b2, b3);
    }
    }
    __syncwarp();
  }
  // row sums across the quad
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  // ---- merge the four warps through shared memory
  __syncthreads();
  float *mo = reinterpret_cast<float *>(smem);   // [WARPS][16][D]
  float *mm = mo + WARPS * 16 * D;               // [WARPS][16]
  float *ml = mm + WARPS * 16;                   // [WARPS][16]
  // int8: n-tile dt holds columns 16 (dt / 2) + 4 q4 + (dt % 2) and +2, in
  // units of 2^-kcur
  // only the G live rows (the query heads of the group) are merged
  const int G = a.G;
  const int oe = (INT8 && kcur != INT_MAX) ? -kcur : 0;
  if (g < G) {
#pragma unroll
    for (int dt = 0; dt < D / 8; dt++) {
      const int d = INT8 ? 16 * (dt >> 1) + 4 * q4 + (dt & 1) : dt * 8 + q4 * 2;
      const int dd = INT8 ? 2 : 1;
      mo[((size_t)warp * 16 + g) * D + d] = INT8 ? mul_pow2f(o[dt][0], oe) : o[dt][0];
      mo[((size_t)warp * 16 + g) * D + d + dd] = INT8 ? mul_pow2f(o[dt][1], oe) : o[dt][1];
    }
    if (q4 == 0) {
      mm[warp * 16 + g] = m0;
      ml[warp * 16 + g] = l0;
    }
  }
  if (g + 8 < G) {
#pragma unroll
    for (int dt = 0; dt < D / 8; dt++) {
      const int d = INT8 ? 16 * (dt >> 1) + 4 * q4 + (dt & 1) : dt * 8 + q4 * 2;
      const int dd = INT8 ? 2 : 1;
      mo[((size_t)warp * 16 + g + 8) * D + d] = INT8 ? mul_pow2f(o[dt][2], oe) : o[dt][2];
      mo[((size_t)warp * 16 + g + 8) * D + d + dd] = INT8 ? mul_pow2f(o[dt][3], oe) : o[dt][3];
    }
    if (q4 == 0) {
      mm[warp * 16 + g + 8] = m1;
      ml[warp * 16 + g + 8] = l1;
    }
  }
  __syncthreads();
  const size_t grp = (size_t)i * a.Hkv + h;
  const float LN2 = 0.69314718055994530942f;
  for (int e = threadIdx.x; e < G * D; e += THREADS) {
    const int r = e / D, d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; w++) M = fmaxf(M, mm[w * 16 + r]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < WARPS; w++) {
        const float f = exp2f(mm[w * 16 + r] - M);
        L += ml[w * 16 + r] * f;
        O += mo[((size_t)w * 16 + r) * D + d] * f;
      }
    }
    if (a.splits == 1) {
      const size_t orow = (size_t)i * a.Hq + (size_t)h * G + r;
      a.out[orow * D + d] = f32_to_bf16_bits(L > 0.f ? O / L : 0.f);
      if (a.lse && d == 0) a.lse[orow] = L > 0.f ? (M + log2f(L)) * LN2 : -INFINITY;
    } else {
      const size_t pr = (grp * a.splits + split) * G + r;
      __stcg(a.ws_o + pr * D + d, O);
      if (d == 0) {
        __stcg(a.ws_ml + pr * 2, M);
        __stcg(a.ws_ml + pr * 2 + 1, L);
      }
    }
  }
  if (a.splits == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(a.counters + grp, 1u) == (unsigned)(a.splits - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int e = threadIdx.x; e < G * D; e += THREADS) {
    const int r = e / D, d = e % D;
    float M = -INFINITY;
    for (int sp = 0; sp < a.splits; sp++) M = fmaxf(M, __ldcg(a.ws_ml + ((grp * a.splits + sp) * G + r) * 2));
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int sp = 0; sp < a.splits; sp++) {
        const size_t pr = (grp * a.splits + sp) * G + r;
        const float f = exp2f(__ldcg(a.ws_ml + pr * 2) - M);
        L += __ldcg(a.ws_ml + pr * 2 + 1) * f;
        O += __ldcg(a.ws_o + pr * D + d) * f;
      }
    }
    const size_t orow = (size_t)i * a.Hq + (size_t)h * G + r;
    a.out[orow * D + d] = f32_to_bf16_bits(L > 0.f ? O / L : 0.f);
    if (a.lse && d == 0) a.lse[orow] = L > 0.f ? (M + log2f(L)) * LN2 : -INFINITY;
  }
  if (threadIdx.x == 0) a.counters[grp] = 0u;
}

template <int D, bool INT8>
int launch_t(vxb_ctx *ctx, const DecodeArgs &a, cudaStream_t st) {
  auto kfn = decode_attn_kernel<D, INT8>;
  using SM = Smem<D, INT8>;
  const size_t merge = (size_t)WARPS * 16 * D * 4 + 2 * WARPS * 16 * 4;
  const size_t smem = SM::TOTAL > merge ? SM::TOTAL : merge;
  static std::atomic<bool> configured[64];  // kernel attributes set on this device (zero-initialized)
  if (!configured[ctx->device & 63]) {
    VXB_CUDA_TRY(ctx, cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    configured[ctx->device & 63] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n * a.Hkv, a.splits);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  VXB_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kfn, a));
  return launch_check(ctx, "decode_attn_kernel");
}

}  // namespace

namespace vxb {

// Token splits per (sequence, kv head). The run time is about the number of
// CTA waves (3 resident CTAs per SM) times the time of one CTA, which is a
// fixed part - pipeline fill and drain, the merge - worth about 300 tokens of
// streaming plus its share of the tokens. Fitted to measurements on B200 (32
// sequences x 8 KV heads: ctx 1k best unsplit, 8k and 32k at 5 splits, 0.96
// and 1.06 of the copy bandwidth; 32 sequences x 32 KV heads at ctx 2k: 2
// splits). At most 12 splits (the merge in the last-arriving CTA grows with
// the split count), at least 64 tokens each.
// VXB_DECODE_SPLITS=n forces n (tuning).
DecodePlan decode_plan(const vxb_ctx *ctx, int n, int Hkv, int max_len) {
  DecodePlan p;
  const int sms = ctx->num_sms > 0 ? ctx->num_sms : 148;
  const long long pairs = (long long)n * Hkv;
  const long long slots = 3LL * sms;
  static const int forced = [] {
    const char *e = std::getenv("VXB_DECODE_SPLITS");
    return e ? std::atoi(e) : 0;
  }();
  auto tps_for = [&](int s) {
    const int t = (max_len + s - 1) / s;
    return max(64, (t + 63) / 64 * 64);
  };
  int best = 1;
  if (forced > 0) {
    best = min(forced, kMaxDecodeSplits);
  } else {
    double best_cost = 1e300;
    for (int s = 1; s <= kMaxDecodeSplits; s++) {
      const int tps = tps_for(s);
      if ((max_len + tps - 1) / tps != s && s > 1) continue;  // the same split count as a smaller s
      const double waves = (double)((pairs * s + slots - 1) / slots);
      const double cost = waves * (300.0 + tps);
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best = s;
      }
    }
  }
  p.tps = tps_for(best);
  p.splits = max(1, (max_len + p.tps - 1) / p.tps);
  return p;
}

size_t decode_ws_bytes(int n, int Hkv, int G, int D, int splits) {
  const size_t pr = (size_t)n * Hkv * splits * G;
  return 256 + pr * D * 4 + pr * 2 * 4 + 256;
}

int decode_attn_launch(vxb_kv *kv, int layer, int n, const int32_t *d_slots, const int32_t *h_slots,
                       const uint16_t *d_q, int Hq, float softmax_scale, uint16_t *d_out, float *d_lse,
                       const DecodePlan &p, float *ws, cudaStream_t st) {
  vxb_ctx *ctx = kv->ctx;
  const int Hkv = kv->num_kv_heads, D = kv->head_dim;
  const int G = Hq / Hkv;
  DecodeArgs a;
  a.q = d_q;
  a.out = d_out;
  a.lse = d_lse;
  a.pool_k = kv->pool_k;
  a.pool_v = kv->pool_v;
  a.sk = kv->scale_k;
  a.sv = kv->scale_v;
  a.tables = kv->d_tables + (size_t)layer * kv->max_seqs * kv->max_blocks_per_seq;
  a.lens = kv->d_lens + (size_t)layer * kv->max_seqs;
  a.slots = d_slots;
  if (!d_slots) {
    if (!h_slots || n > kMaxInlineRows) return set_error(ctx, VXB_EINVAL, "decode attention: %d rows without device slots", n);
    for (int i = 0; i < n; i++) a.slots_inline[i] = h_slots[i];
  }
  const size_t pr = (size_t)n * Hkv * p.splits * G;
  a.ws_ml = ws;
  a.ws_o = ws + ((pr * 2 + 63) / 64 * 64);
  a.counters = ctx->counters;
  a.n = n;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = G;
  a.bs = kv->block_size;
  a.mbps = kv->max_blocks_per_seq;
  a.splits = p.splits;
  a.tps = p.tps;
  a.scale_log2 = softmax_scale * 1.44269504088896340736f;
  const bool i8 = kv->dtype == VXB_I8;
  if (D == 128) return i8 ? launch_t<128, true>(ctx, a, st) : launch_t<128, false>(ctx, a, st);
  return i8 ? launch_t<64, true>(ctx, a, st) : launch_t<64, false>(ctx, a, st);
}

}  // namespace vxb

VXB_API int vxb_decode_attention(vxb_kv *kv, int layer, int n, const int64_t *h_seq_ids, const uint16_t *d_q,
                                 int num_q_heads, float softmax_scale, uint16_t *d_out, float *d_lse, void *stream) {
  if (!kv || !kv->ctx) return set_error(nullptr, VXB_EINVAL, "vxb_decode_attention: null cache");
  vxb_ctx *ctx = kv->ctx;
  if (layer < 0 || layer >= kv->num_layers) return set_error(ctx, VXB_EINVAL, "vxb_decode_attention: layer out of range");
  if (n < 0 || (n > 0 && (!h_seq_ids || !d_q || !d_out))) return set_error(ctx, VXB_EINVAL, "vxb_decode_attention: bad arguments");
  if (num_q_heads <= 0 || num_q_heads % kv->num_kv_heads || num_q_heads / kv->num_kv_heads > 16)
    return set_error(ctx, VXB_EINVAL, "vxb_decode_attention: num_q_heads %d must be a multiple (<= 16x) of the %d kv heads",
                     num_q_heads, kv->num_kv_heads);
  if (((uintptr_t)d_q) % 16) return set_error(ctx, VXB_EINVAL, "vxb_decode_attention: q must be 16-byte aligned");
  if (n == 0) return VXB_OK;
  if (int rc = use_device(ctx)) return rc;
  std::vector<int32_t> slots(n);
  int max_len = 0;
  for (int i = 0; i < n; i++) {
    auto si = kv->slot_of.find(h_seq_ids[i]);
    slots[i] = si == kv->slot_of.end() ? -1 : si->second;
    auto it = kv->tables.find(std::make_pair(layer, h_seq_ids[i]));
    if (it != kv->tables.end()) max_len = std::max<int>(max_len, (int)it->second.len);
  }
  const int G = num_q_heads / kv->num_kv_heads;
  const int rows = std::min(n, kMaxInlineRows);
  const DecodePlan p = decode_plan(ctx, rows, kv->num_kv_heads, std::max(max_len, 1));
  const size_t wsb = decode_ws_bytes(rows, kv->num_kv_heads, G, kv->head_dim, p.splits);
  if (int rc = ws_reserve(ctx, wsb, (size_t)rows * kv->num_kv_heads)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  // rows go in chunks whose slot ids travel as kernel parameters
  for (int r0 = 0; r0 < n; r0 += kMaxInlineRows) {
    const int nr = std::min(kMaxInlineRows, n - r0);
    const size_t off = (size_t)r0 * num_q_heads * kv->head_dim;
    if (int rc = decode_attn_launch(kv, layer, nr, nullptr, slots.data() + r0, d_q + off, num_q_heads, softmax_scale,
                                    d_out + off, d_lse ? d_lse + (size_t)r0 * num_q_heads : nullptr, p,
                                    (float *)ctx->ws, st))
      return rc;
  }
  return VXB_OK;
}
