// K3: flash-attention forward on the 5th-generation tensor cores (tcgen05).
//
//   O[b, i, h, :] = sum_j softmax_j(scale * q_i . k_j  (j <= i if causal)) v_j
//   lse[b, h, i]  = log sum_j exp(scale * q_i . k_j)
//
// Replaces flash_attention_forward / multi_head_flash_attention
// (src/flash_attention.rs:53-159, 519-564). Inputs are [B, S, H, d] bf16 (per
// batch the reference's [N, H*d] rows with the heads interleaved,
// src/flash_attention.rs:545-551), d = 128; grouped K/V heads (Hkv | H).
//
// One CTA per (128-query tile, head, batch), 6 warps:
//  * warp 5 (one elected thread) loads Q once and the K and V tiles of 128
//    keys into two separate 3-stage rings with TMA (4-D tensor maps, 128-byte
//    swizzle); a K stage is refilled as soon as its S = Q K^T has completed,
//    a V stage once its P.V has.
//  * warp 4 (one elected thread) issues the MMAs: S = Q K^T (M=128, N=128,
//    K=128 as 8 x K16) into TMEM columns [0,128), then O += P V with A = P
//    read from TMEM and B = V read MN-major from shared memory, into TMEM
//    columns [128,256). Completion is signalled to mbarriers with
//    tcgen05.commit.
//  * warps 0-3 own one query row each (TMEM lane = row): they read the row of
//    S with tcgen05.ld, apply scale (log2 domain) and the causal / length mask,
//    keep a reference max m and the sum l, and store P = 2^(s - m) as bf16
//    hi + lo with tcgen05.st into one of two TMEM P buffers (columns
//    [256,384) and [384,512)), so the exponentials of tile j+1 need not wait
//    for the P.V of tile j. m moves (and the row of O in TMEM is rescaled)
//    only when the row's max exceeds it by more than 2^8, so most tiles skip
//    the rescale.
//  * The MMA of S for the next tile is issued as soon as the softmax warps have
//    read the current S, so it overlaps their exponentials.
// Every mbarrier wait is bounded (clock64); a timeout sets the context's
// device error word and the kernel runs to completion. No multicast.
#include <atomic>
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

#include "tc_common.h"
#include "vxb_internal.h"

using namespace vxb;
using namespace vxb::tc;

namespace {

constexpr int D = 128;        // head dim
constexpr int BM = 128;       // queries per CTA
constexpr int BN = 128;       // keys per tile
constexpr int THREADS = 192;  // 4 softmax warps + MMA warp + TMA warp
constexpr int TILE_BYTES = BM * D * 2;  // 32 KB: two 64-column slabs of [128 rows x 128 B]
constexpr int SLAB = 128 * 128;         // bytes of one slab
constexpr int KV_STAGES = 3;
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE_BYTES;                  // KV_STAGES stages
constexpr int OFF_V = OFF_K + KV_STAGES * TILE_BYTES;      // KV_STAGES stages
constexpr int SMEM_BYTES = OFF_V + KV_STAGES * TILE_BYTES;  // 224 KB
constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;              // + alignment slack
// TMEM columns: S [0,128), O [128,256), P buffers [256,384) and [384,512),
// each P = bf16 hi (64 columns of key pairs) then lo (64 columns)
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_O = 128, COL_P = 256;
// O is rescaled only when a row's running max grows by more than this (log2
// units): P then stays below 2^8, exact in f32 and representable in bf16.
constexpr float RESCALE_THRESHOLD = 8.f;

struct FlashArgs {
  uint16_t *o;
  float *lse;
  int *err;
  int B, H, Hkv, S, n_qtiles;
  float scale_log2;
};

struct Bars {
  uint64_t q, k_full[KV_STAGES], k_empty[KV_STAGES], v_full[KV_STAGES], v_empty[KV_STAGES], s_full, s_free, p_full,
      o_done, p_free[2];
};

template <bool CAUSAL>
__global__ void __launch_bounds__(THREADS, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, const FlashArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) Bars bars;
  __shared__ uint32_t tmem_base_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = a.n_qtiles - 1 - (int)blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (a.H / a.Hkv);
  const int q0 = qt * BM;
  const int kv_tiles = (a.S + BN - 1) / BN;
  const int n_kv = CAUSAL ? min(qt + 1, kv_tiles) : kv_tiles;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 32) {
    mbar_init(&bars.q, 1);
    for (int i = 0; i < KV_STAGES; i++) {
      mbar_init(&bars.k_full[i], 1);
      mbar_init(&bars.k_empty[i], 1);
      mbar_init(&bars.v_full[i], 1);
      mbar_init(&bars.v_empty[i], 1);
    }
    mbar_init(&bars.s_full, 1);
    mbar_init(&bars.s_free, 4);
    mbar_init(&bars.p_full, 4);
    mbar_init(&bars.o_done, 1);
    mbar_init(&bars.p_free[0], 1);
    mbar_init(&bars.p_free[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  const uint32_t tS = tmem, tO = tmem + COL_O;

  if (warp == 5) {
    // ---------------- TMA producer: Q once, then K and V of each key tile into
    // their own rings. K(j) waits only for S(j-3), V(j) for PV(j-3), so K
    // tiles run ahead of the P.V products.
    if (lane == 0) {
      mbar_expect_tx(&bars.q, TILE_BYTES);
      tma_load_4d(sm + OFF_Q, &tq, 0, h, q0, b, &bars.q);
      tma_load_4d(sm + OFF_Q + SLAB, &tq, 64, h, q0, b, &bars.q);
      for (int j = 0; j < n_kv; j++) {
        const int st = j % KV_STAGES;
        const uint32_t ph = ((j / KV_STAGES) - 1) & 1;
        uint8_t *k = sm + OFF_K + st * TILE_BYTES, *v = sm + OFF_V + st * TILE_BYTES;
        if (j >= KV_STAGES) wait_or_flag(&bars.k_empty[st], ph, a.err);
        mbar_expect_tx(&bars.k_full[st], TILE_BYTES);
        tma_load_4d(k, &tk, 0, hk, j * BN, b, &bars.k_full[st]);
        tma_load_4d(k + SLAB, &tk, 64, hk, j * BN, b, &bars.k_full[st]);
        if (j >= KV_STAGES) wait_or_flag(&bars.v_empty[st], ph, a.err);
        mbar_expect_tx(&bars.v_full[st], TILE_BYTES);
        tma_load_4d(v, &tv, 0, hk, j * BN, b, &bars.v_full[st]);
        tma_load_4d(v + SLAB, &tv, 64, hk, j * BN, b, &bars.v_full[st]);
      }
    }
    __syncwarp();
  } else if (warp == 4) {
    // ---------------- MMA issue (one thread): S(j) then PV(j-1)
    if (lane == 0) {
      const uint32_t sQ = smem_u32(sm + OFF_Q);
      constexpr uint32_t ID_QK = idesc_bf16(BM, BN, false), ID_PV = idesc_bf16(BM, D, true);
      wait_or_flag(&bars.q, 0, a.err);
      auto issue_pv = [&](int j) {
        const int st = j % KV_STAGES;
        wait_or_flag(&bars.p_full, j & 1, a.err);
        wait_or_flag(&bars.v_full[st], (j / KV_STAGES) & 1, a.err);
        tc_fence_after();
        const uint32_t sV = smem_u32(sm + OFF_V + st * TILE_BYTES);
        const uint32_t tP = tmem + COL_P + (uint32_t)(j & 1) * 128;
        // O += P_hi V + P_lo V: the K dimension runs over the keys twice
#pragma unroll
        for (int t = 0; t < 2 * BN / 16; t++) {
          const int tk = t & 7;
          // A = P from TMEM: 16 keys = 8 columns of bf16 pairs (hi, then lo)
          // B = V read MN-major: 16 keys = two 8-row groups of 1024 bytes; the
          // two 64-column slabs of d are 16 KB apart
          const uint64_t bd = sw128_desc(sV + tk * 2048, SLAB, 1024);
          umma_bf16_ts(tO, tP + (uint32_t)t * 8, bd, ID_PV, (j > 0 || t > 0) ? 1u : 0u);
        }
        umma_commit(&bars.o_done);
        umma_commit(&bars.v_empty[st]);
        umma_commit(&bars.p_free[j & 1]);
      };
      for (int j = 0; j < n_kv; j++) {
        const int st = j % KV_STAGES;
        wait_or_flag(&bars.k_full[st], (j / KV_STAGES) & 1, a.err);
        if (j > 0) wait_or_flag(&bars.s_free, (j - 1) & 1, a.err);
        tc_fence_after();
        const uint32_t sK = smem_u32(sm + OFF_K + st * TILE_BYTES);
#pragma unroll
        for (int t = 0; t < D / 16; t++) {
          const uint32_t off = (t >> 2) * SLAB + (t & 3) * 32;
          umma_bf16(tS, sw128_desc(sQ + off, 16, 1024), sw128_desc(sK + off, 16, 1024), ID_QK, t > 0 ? 1u : 0u);
        }
        umma_commit(&bars.s_full);
        umma_commit(&bars.k_empty[st]);
        if (j > 0) issue_pv(j - 1);
      }
      issue_pv(n_kv - 1);
    }
    __syncwarp();
  } else {
    // ---------------- softmax: thread r owns query row q0 + r (TMEM lane r)
    const int r = threadIdx.x;
    const int row = q0 + r;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const int lim = CAUSAL ? min(a.S - 1, row) : a.S - 1;  // last visible key
    // m: the reference max of the row (log2 domain), P = 2^(s - m) <= 2^8
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < n_kv; j++) {
      wait_or_flag(&bars.s_full, j & 1, a.err);
      tc_fence_after();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; c++) tmem_ld32(tS + lane_off + c * 32, *reinterpret_cast<float(*)[32]>(s + c * 32));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.s_free);

      const int k0 = j * BN;
      float mx = -INFINITY;
      if (k0 + BN - 1 <= lim) {
#pragma unroll
        for (int c = 0; c < BN; c++) mx = fmaxf(mx, s[c]);
      } else {
#pragma unroll
        for (int c = 0; c < BN; c++) {
          s[c] = (k0 + c <= lim) ? s[c] : -INFINITY;
          mx = fmaxf(mx, s[c]);
        }
      }
      mx *= a.scale_log2;
      // move the reference max only when the row's max outgrows it by more
      // than the threshold (or the row had no visible key yet)
      const bool grow = mx > m + RESCALE_THRESHOLD;
      const float m_new = grow ? mx : m;
      const float mb = m_new == -INFINITY ? 0.f : m_new;  // rows with no visible key yet
      const float alpha = grow ? ex2(m - mb) : 1.f;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < BN; c++) {
        const float p = ex2(fmaf(s[c], a.scale_log2, -mb));
        s[c] = p;
        sum += p;
      }
      l = l * alpha + sum;
      m = m_new;

      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // O holds the tiles before j: wait for the last P.V, then rescale the
        // rows whose reference max moved
        wait_or_flag(&bars.o_done, (j - 1) & 1, a.err);
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; c++) {
          float o[32];
          tmem_ld32(tO + lane_off + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i++) o[i] *= alpha;
          tmem_st32(tO + lane_off + c * 32, o);
        }
        tmem_wait_st();
      }
      // P buffer j % 2 is free once P.V of tile j - 2 has completed
      if (j >= 2) {
        wait_or_flag(&bars.p_free[j & 1], ((j >> 1) - 1) & 1, a.err);
        tc_fence_after();
      }
      // P as bf16 hi + lo (p - hi rounded again: 16 significant bits, so the
      // P.V product keeps the precision of the f32 softmax) into the row's
      // TMEM lane: key pairs (2c, 2c+1) in column c, hi in columns 0-63, lo
      // in columns 64-127
      const uint32_t tP = tmem + COL_P + (uint32_t)(j & 1) * 128 + lane_off;
#pragma unroll
      for (int c = 0; c < BN / 64; c++) {
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int e = 0; e < 32; e++) {
          const float p0 = s[c * 64 + 2 * e], p1 = s[c * 64 + 2 * e + 1];
          hi[e] = pack_bf16(p0, p1);
          lo[e] = pack_bf16(p0 - __uint_as_float(hi[e] << 16), p1 - __uint_as_float(hi[e] & 0xFFFF0000u));
        }
        tmem_st32u(tP + c * 32, hi);
        tmem_st32u(tP + 64 + c * 32, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.p_full);
    }
    // ---------------- epilogue: O / l (bf16) and lse (natural log)
    wait_or_flag(&bars.o_done, (n_kv - 1) & 1, a.err);
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const bool live = row < a.S;
    uint16_t *orow = a.o + (((size_t)b * a.S + (live ? row : 0)) * a.H + h) * D;
#pragma unroll
    for (int c = 0; c < D / 32; c++) {
      float o[32];
      tmem_ld32(tO + lane_off + c * 32, o);
      tmem_wait_ld();
      if (live) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          uint4 w;
          w.x = pack_bf16(o[q * 8 + 0] * inv, o[q * 8 + 1] * inv);
          w.y = pack_bf16(o[q * 8 + 2] * inv, o[q * 8 + 3] * inv);
          w.z = pack_bf16(o[q * 8 + 4] * inv, o[q * 8 + 5] * inv);
          w.w = pack_bf16(o[q * 8 + 6] * inv, o[q * 8 + 7] * inv);
          *reinterpret_cast<uint4 *>(orow + c * 32 + q * 8) = w;
        }
      }
    }
    if (live && a.lse) a.lse[((size_t)b * a.H + h) * a.S + row] = l > 0.f ? (m + __log2f(l)) * 0.69314718055994531f : -INFINITY;
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
}

// ---------------- host: tensor maps through the driver entry point
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
      set_error(ctx, VXB_ECUDA, "vxb_flash_fwd: cuTensorMapEncodeTiled is not available from the driver");
      return nullptr;
    }
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// [B, S, heads, 128] bf16 -> 4-D map (d, head, s, b), box (64, 1, box_rows, 1)
int make_map(vxb_ctx *ctx, EncodeTiledFn fn, CUtensorMap *map, const void *base, int B, int S, int heads,
             int box_rows) {
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)heads * D * 2, (cuuint64_t)S * heads * D * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ctx, VXB_EINVAL, "vxb_flash_fwd: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VXB_OK;
}

template <bool CAUSAL>
int launch(vxb_ctx *ctx, const CUtensorMap &q, const CUtensorMap &k, const CUtensorMap &v, const FlashArgs &a,
           cudaStream_t st) {
  static std::atomic<bool> configured[64];  // kernel attributes set on this device (zero-initialized)
  const int dev = ctx->device & 63;
  if (!configured[dev]) {
    VXB_CUDA_TRY(ctx, cudaFuncSetAttribute(flash_fwd_kernel<CAUSAL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           SMEM_ALLOC));
    configured[dev] = true;
  }
  dim3 grid(a.n_qtiles, a.H, a.B);
  flash_fwd_kernel<CAUSAL><<<grid, THREADS, SMEM_ALLOC, st>>>(q, k, v, a);
  return launch_check(ctx, "flash_fwd_kernel");
}

}  // namespace

VXB_API int vxb_flash_fwd(vxb_ctx *ctx, const uint16_t *d_q, const uint16_t *d_k, const uint16_t *d_v, int B, int H,
                          int Hkv, int S, int d, float scale, int causal, uint16_t *d_o, float *d_lse, void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_flash_fwd: null context");
  if (d != D) return set_error(ctx, VXB_EUNSUPPORTED, "vxb_flash_fwd: head_dim %d (only 128 is implemented)", d);
  if (B < 1 || H < 1 || Hkv < 1 || S < 1 || H % Hkv)
    return set_error(ctx, VXB_EINVAL, "vxb_flash_fwd: bad shape B=%d H=%d Hkv=%d S=%d", B, H, Hkv, S);
  if (!d_q || !d_k || !d_v || !d_o) return set_error(ctx, VXB_EINVAL, "vxb_flash_fwd: null pointer");
  if (((uintptr_t)d_q | (uintptr_t)d_k | (uintptr_t)d_v | (uintptr_t)d_o) % 16)
    return set_error(ctx, VXB_EINVAL, "vxb_flash_fwd: tensors must be 16-byte aligned");
  if (!(scale > 0.f)) return set_error(ctx, VXB_EINVAL, "vxb_flash_fwd: scale must be positive");
  if (int rc = use_device(ctx)) return rc;
  if (int rc = ws_reserve(ctx, 0, 0)) return rc;  // device error word
  EncodeTiledFn fn = encode_fn(ctx);
  if (!fn) return VXB_ECUDA;
  CUtensorMap mq, mk, mv;
  if (int rc = make_map(ctx, fn, &mq, d_q, B, S, H, BM)) return rc;
  if (int rc = make_map(ctx, fn, &mk, d_k, B, S, Hkv, BN)) return rc;
  if (int rc = make_map(ctx, fn, &mv, d_v, B, S, Hkv, BN)) return rc;
  FlashArgs a;
  a.o = d_o;
  a.lse = d_lse;
  a.err = ctx->d_err;
  a.B = B;
  a.H = H;
  a.Hkv = Hkv;
  a.S = S;
  a.n_qtiles = (S + BM - 1) / BM;
  a.scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t st = (cudaStream_t)stream;
  return causal ? launch<true>(ctx, mq, mk, mv, a, st) : launch<false>(ctx, mq, mk, mv, a, st);
}
