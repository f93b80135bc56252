// K1 batches 9-32 on the 5th-generation tensor cores (tcgen05): the skinny
// GEMM y[b, n] = sum_k deq(W)[n, k] x[b, k] with the quantized codes decoded
// into tensor memory as the MMA's A operand. Opt-in (VXB_GEMV_TCGEN05=1)
// until it is faster than the group-CTA kernel of gemv.cu.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>

#include <cooperative_groups.h>

#include "gemv.h"
#include "gemv_common.h"
#include "tc_common.h"

using namespace vxb;
namespace cg = cooperative_groups;

namespace {

// Batches 9-32: tcgen05 skinny GEMM.
//
// A CTA owns one 128-row group (8 sixteen-row tiles) and a k-range of whole
// weight stages. A stage is one pair of 64-column steps (2 chunks of each tile
// for Q4_0, 4 for Q8_0) plus the pair's x boxes, in one ring slot with one
// mbarrier. Per step the group's codes become the A operand of tcgen05.mma in
// tensor memory: exact small integers as bf16, written with
// tcgen05.st.16x256b, whose register layout (thread t: lanes t/4 and t/4+8,
// columns 2(t%4) and 2(t%4)+1) is the m16n8k16 A fragment the tiled units
// already hold, the units' k permutation lining the fragment up with the
// matrix columns. x is the B operand: one 2-D TMA box per step [NB rows x 64
// columns], 128-byte swizzled, K-major (rows past the batch and columns past
// K arrive as zeros). Each 32-column block accumulates into its own NB TMEM
// columns (two M=128 x N=NB x K=16 MMAs), and the epilogue multiplies the
// block's f32 sums by the f16 block scales (acc += d * D): the scales never
// round into an operand.
//
// Eight worker warps run every pair in lockstep, and a ninth warp issues the
// MMAs and the TMA refills. Per pair, worker warp w reads the codes of tile
// 2(w%4) + w/4 for both steps, runs the epilogue of the previous pair (block
// w/4 of both steps for the 32 rows of its quadrant: one tcgen05.ld per step
// and packed f32x2 FMAs), decodes and stores its codes into the A buffer,
// and the nine warps meet on a hardware named barrier (sleeping, no
// polling). The MMA warp then refills the ring slot of the previous pair
// (whose MMAs the workers saw complete in their epilogue) and issues this
// pair's eight MMAs with one commit, while the workers move on to the next
// pair - so no worker waits for the MMA issue at the next barrier (with a
// worker thread issuing them, that wait was the kernel's largest stall). A
// and the accumulators have one buffer each (192 of 256 TMEM columns, two
// CTAs per SM): the epilogue of the previous pair waits for its MMAs before
// the A buffer is rewritten, and the next MMAs are issued only after every
// worker has read the accumulators. The first stages' weights are requested
// before the wait for the kernel that produces x.
// S > 1 CTAs of a row group form a cluster and add their partial sums through
// distributed shared memory in CTA order.
constexpr int TC_WORKERS = 256;                 // eight worker warps
constexpr int TC_THREADS = TC_WORKERS + 32;     // + the MMA / TMA warp
constexpr int TC_MAX_WR = 8;
constexpr uint32_t TC_COLS = 256, TC_ACOL = 0, TC_DCOL = 64;
constexpr size_t TC_SMEM_CAP = 110 * 1024;  // two CTAs per SM
constexpr size_t TC_SMEM_MIN = 80 * 1024;   // and never three (each holds 256 TMEM columns)

struct TcArgs {
  const uint8_t *units;  // unit (tile 0, chunk 0)
  const uint32_t *hdr;
  void *y;
  const float *resid;  // optional f32 [B, N]
  int *err;
  int N, K, B, n_chunks, y_dtype;
  int wr;     // ring slots
  int n_wst;  // stages over the padded k range
  int S;      // CTAs per row group (cluster along y)
};

template <int FMT>
struct TcGeo {
  static constexpr int UNIT = Geo<FMT>::UNIT;
  static constexpr int CPS = FMT == 0 ? 2 : 4;  // chunks per stage (= 2 steps of 64 columns)
  static constexpr int TBYTES = CPS * UNIT;      // one tile's part of a stage
  static constexpr int WSB = 8 * TBYTES;         // weights of a stage
};

template <int FMT, int NB>
struct TcSmem {
  static constexpr int XB = NB * 128;  // one x box
  static constexpr int SLOT = (2 * XB + TcGeo<FMT>::WSB + 1023) / 1024 * 1024;
  __host__ __device__ static size_t red_off(int wr) { return (size_t)wr * SLOT; }
  __host__ __device__ static size_t bytes(int wr) {
    const size_t b = red_off(wr) + (size_t)NB * 128 * 4 + 1024;  // + 1024: base alignment
    return b < TC_SMEM_MIN ? TC_SMEM_MIN : b;
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

// Bounded wait by all lanes of a warp with a warp-uniform outcome; a failure
// is recorded once (the kernel then runs to its end on whatever the buffers
// hold, so every thread still meets every barrier).
__device__ __forceinline__ void tc_wait_warp(uint64_t *bar, uint32_t parity, int *err) {
  const bool mine = mbar_wait(bar, parity);
  if (!__all_sync(0xffffffffu, mine) && (threadIdx.x & 31) == 0) atomicExch(err, 1);
}

// the worker warps and the MMA warp, once per pair: the A buffer is written
__device__ __forceinline__ void pair_sync() { asm volatile("bar.sync 1, %0;" ::"n"(TC_THREADS) : "memory"); }
// the worker warps only
__device__ __forceinline__ void workers_sync() { asm volatile("bar.sync 2, %0;" ::"n"(TC_WORKERS) : "memory"); }

// The 16x256b.x4 registers of one tile for one 64-column step: k16 step s
// holds {row g: k 4q..4q+1, row g: 4q+2..4q+3, row g+8: 4q..4q+1, row g+8:
// 4q+2..4q+3} = fragment pairs {a0a1, a4a5, a2a3, a6a7}.
template <int FMT>
__device__ __forceinline__ void tc_decode_words(const uint4 c0, const uint4 c1, uint32_t (&r)[16]) {
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

template <int FMT, int NB>
__global__ void __launch_bounds__(TC_THREADS, 2)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                   const TcArgs a) {
  using TG = TcGeo<FMT>;
  using SM = TcSmem<FMT, NB>;
  constexpr int UNIT = TG::UNIT, TBYTES = TG::TBYTES, CPS = TG::CPS;
  constexpr uint32_t STAGE_TX = (uint32_t)(TG::WSB + 2 * SM::XB);
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  float *red = reinterpret_cast<float *>(sm + SM::red_off(a.wr));  // [NB][128]
  __shared__ __align__(8) uint64_t wfull[TC_MAX_WR], mdone[2];
  __shared__ uint32_t tmem_base_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, half = warp >> 2;
  const int grp = blockIdx.x;
  const int ws0 = (int)((long long)blockIdx.y * a.n_wst / a.S);
  const int nws = (int)((long long)(blockIdx.y + 1) * a.n_wst / a.S) - ws0;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(TC_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.wr; i++) mbar_init(&wfull[i], 1);
    mbar_init(&mdone[0], 1);
    mbar_init(&mdone[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  vxb::tc::tc_fence_before();
  __syncthreads();
  vxb::tc::tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  asm volatile("griddepcontrol.launch_dependents;");

  // stage ws of this CTA into ring slot `slot`: the weights (one 3-D box of 8
  // tiles x CPS chunks) and the x boxes of its two steps
  auto load_weights = [&](int ws, int slot) {
    uint8_t *d = sm + (size_t)slot * SM::SLOT;
    mbar_expect_tx(&wfull[slot], STAGE_TX);
    vxb::tc::tma_load_3d(d + 2 * SM::XB, &wmap, 0, (ws0 + ws) * CPS, grp * 8, &wfull[slot]);
  };
  auto load_x = [&](int ws, int slot) {
    uint8_t *d = sm + (size_t)slot * SM::SLOT;
    vxb::tc::tma_load_2d(d, &xmap, (ws0 + ws) * 128, 0, &wfull[slot]);
    vxb::tc::tma_load_2d(d + SM::XB, &xmap, (ws0 + ws) * 128 + 64, 0, &wfull[slot]);
  };
  if (threadIdx.x == TC_WORKERS) {
    const int pre = min(a.wr, nws);
    for (int ws = 0; ws < pre; ws++) load_weights(ws, ws);
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x comes from the previous kernel
    for (int ws = 0; ws < pre; ws++) load_x(ws, ws);
  }
  constexpr uint32_t ID = vxb::tc::idesc_bf16(128, NB, false);
  const int nsteps = 2 * nws;  // 64-column steps, two per stage
  if (warp == 8) {
    // ---- the MMA / TMA warp (thread TC_WORKERS): once the workers have stored
    // step i's codes in A buffer i % 2, issue its four MMAs into accumulator
    // buffer i % 2 and commit them to mdone[i % 2]; at the first step of a
    // stage, wait for the previous stage's last MMAs and refill its slot
    int slot = 0;
    for (int ws = 0; ws < nws; ws++) {
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const int i = 2 * ws + j;
        pair_sync();
        if (lane == 0) {
          vxb::tc::tc_fence_after();
          const uint32_t xa = smem_u32(sm + (size_t)slot * SM::SLOT);
#pragma unroll
          for (int b = 0; b < 2; b++)
#pragma unroll
            for (int k = 0; k < 2; k++)
              vxb::tc::umma_bf16_ts(tmem + TC_DCOL + (uint32_t)(j * 2 + b) * NB,
                                    tmem + TC_ACOL + j * 32 + (2 * b + k) * 8,
                                    vxb::tc::sw128_desc(xa + j * SM::XB + (2 * b + k) * 32, 16, 1024), ID, k);
          vxb::tc::umma_commit(&mdone[j]);
          if (j == 0 && i >= 2) {
            // step i - 1 (odd: mdone[1], its (i - 1) / 2-th phase) was the
            // last reader of the previous stage's slot
            vxb::tc::wait_or_flag(&mdone[1], ((i - 1) >> 1) & 1, a.err);
            const int pslot = slot == 0 ? a.wr - 1 : slot - 1;
            if (ws - 1 + a.wr < nws) {
              load_weights(ws - 1 + a.wr, pslot);
              load_x(ws - 1 + a.wr, pslot);
            }
          }
        }
        __syncwarp();
      }
      if (++slot == a.wr) slot = 0;
    }
  } else {  // ---- the eight worker warps

  const bool subn = (__ldg(a.hdr + 1) & TILED_FLAG_SUBNORMAL_SCALES) != 0;
  // epilogue row of this thread: 32q + lane = tile je, row pair pi, half ph
  const int je = 2 * q + (lane >> 4), pi = (lane & 15) & 7, ph = (lane & 15) >> 3;
  const int dtile = 2 * q + half;  // the tile this warp decodes
  const uint32_t tq = (uint32_t)(32 * q) << 16;  // TMEM lane base of the quadrant
  float2 acc[NB / 2];
#pragma unroll
  for (int n = 0; n < NB / 2; n++) acc[n] = make_float2(0.f, 0.f);

  // epilogue of step i: block `half` of the step, rows of quadrant q, in
  // accumulator buffer i % 2 (packed f32x2 FMAs; the blocks add in step order)
  auto epilogue = [&](int i, float sc) {
    tc_wait_warp(&mdone[i & 1], (i >> 1) & 1, a.err);
    vxb::tc::tc_fence_after();
    float v[NB];
    tmem_ld_nb<NB>(tmem + TC_DCOL + (uint32_t)((i & 1) * 2 + half) * NB + tq, v);
    vxb::tc::tmem_wait_ld();
    vxb::tc::tc_fence_before();
#pragma unroll
    for (int n = 0; n < NB / 2; n++) acc[n] = __ffma2_rn(make_float2(v[2 * n], v[2 * n + 1]), make_float2(sc, sc), acc[n]);
  };

  // Step i writes A buffer i % 2 and accumulator buffer i % 2; the epilogue
  // of step i - 1 runs after step i's barrier, while the tensor core works
  // on step i. A buffer i % 2 is free again once step i - 2's MMAs are
  // complete (the epilogue of step i - 2 waited for them).
  float s_prev = 0.f;  // scale of the previous step's block for this thread's row
  int slot = 0;
  uint32_t par = 0;
  constexpr int NU = FMT == 0 ? 2 : 4;
  uint4 cw[NU];  // this warp's tile codes of the current stage (raw)
  for (int ws = 0; ws < nws; ws++) {
    tc_wait_warp(&wfull[slot], par, a.err);
    const uint8_t *wst = sm + (size_t)slot * SM::SLOT + 2 * SM::XB;
    {
      const uint8_t *tu = wst + dtile * TBYTES + lane * 16;
#pragma unroll
      for (int u = 0; u < NU; u++) cw[u] = *reinterpret_cast<const uint4 *>(tu + u * UNIT);
    }
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int i = 2 * ws + j;
      float sc;
      {
        // the f16 scale of block `half` of step j for this thread's row
        const uint8_t *ue = wst + je * TBYTES + 512;
        uint32_t w;
        if (FMT == 0) {
          const uint2 t2 = *reinterpret_cast<const uint2 *>(ue + j * UNIT + pi * 8);
          w = half ? t2.y : t2.x;
        } else {
          w = *reinterpret_cast<const uint32_t *>(ue + (2 * j + half) * UNIT + pi * 4);
        }
        const float2 d = decode_scales(w, subn);
        sc = ph ? d.y : d.x;
      }
      {
        uint32_t r[16];
        if (FMT == 0)
          tc_decode_words<FMT>(cw[j], cw[j], r);
        else
          tc_decode_words<FMT>(cw[2 * j], cw[2 * j + 1], r);
        tmem_st_16x256b_x4(tmem + TC_ACOL + 32 * j + ((uint32_t)(32 * q + 16 * half) << 16), r);
      }
      vxb::tc::tmem_wait_st();
      vxb::tc::tc_fence_before();
      pair_sync();
      if (i > 0) epilogue(i - 1, s_prev);
      s_prev = sc;
    }
    if (++slot == a.wr) {
      slot = 0;
      par ^= 1u;
    }
  }
  if (nsteps > 0) epilogue(nsteps - 1, s_prev);

  // rows of quadrant q: block-0 warps (half 0) and block-1 warps (half 1) add
  asm volatile("griddepcontrol.wait;" ::: "memory");  // before any global write of this thread
  const int rr = 32 * q + lane;
  if (half == 1)
#pragma unroll
    for (int n = 0; n < NB / 2; n++) {
      red[(2 * n) * 128 + rr] = acc[n].x;
      red[(2 * n + 1) * 128 + rr] = acc[n].y;
    }
  workers_sync();
  if (half == 0) {
    float v[NB];
#pragma unroll
    for (int n = 0; n < NB / 2; n++) {
      v[2 * n] = acc[n].x + red[(2 * n) * 128 + rr];
      v[2 * n + 1] = acc[n].y + red[(2 * n + 1) * 128 + rr];
    }
    const int row = grp * 128 + rr;
    if (a.S == 1) {
      if (row < a.N)
#pragma unroll
        for (int n = 0; n < NB; n++) {
          if (n >= a.B) break;
          const size_t o = (size_t)n * a.N + row;
          float y = v[n];
          if (a.resid) y += __ldcg(a.resid + o);
          if (a.y_dtype == VXB_BF16)
            ((uint16_t *)a.y)[o] = f32_to_bf16_bits(y);
          else
            ((float *)a.y)[o] = y;
        }
    } else {
#pragma unroll
      for (int n = 0; n < NB; n++) red[n * 128 + rr] = v[n];
    }
  }

  }  // worker warps

  if (a.S > 1) {
    // ---- the S CTAs of the row group: CTA c sums a slice of the outputs over
    // the peers in CTA order; nobody exits before all reads are done
    cluster_sync_all();
    cg::cluster_group cl = cg::this_cluster();
    const int nout = a.B * 128;
    const int per = (nout + a.S - 1) / a.S;
    const int i1 = min(nout, ((int)blockIdx.y + 1) * per);
    for (int i = (int)blockIdx.y * per + threadIdx.x; i < i1; i += TC_THREADS) {
      const int n = i >> 7, r2 = i & 127;
      float y = 0.f;
      for (int c = 0; c < a.S; c++) y += *cl.map_shared_rank(red + n * 128 + r2, (unsigned)c);
      const int row = grp * 128 + r2;
      if (row < a.N) {
        const size_t o = (size_t)n * a.N + row;
        if (a.resid) y += __ldcg(a.resid + o);
        if (a.y_dtype == VXB_BF16)
          ((uint16_t *)a.y)[o] = f32_to_bf16_bits(y);
        else
          ((float *)a.y)[o] = y;
      }
    }
    cluster_sync_all();
  }
  vxb::tc::tc_fence_before();
  __syncthreads();
  vxb::tc::tc_fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_COLS));
}

struct TcPlan {
  int S = 0, wr = 0, n_wst = 0;
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
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM_CAP) == cudaSuccess) {
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

// k-splits S and ring depth: two CTAs per SM (the shared-memory cap and the
// 256 TMEM columns each). A CTA's time is its stage count times a per-stage
// cost that grows when two CTAs share an SM, so the plan spreads the row
// groups' stages over every SM: the busiest SM's stages (CTAs spread evenly,
// a second wave counted whole), plus about 0.7 us for a cluster reduction.
// The co-residency of clusters is taken from the plain per-SM occupancy (the
// cluster occupancy query reports fewer co-resident clusters of 3 than run
// in one wave in practice: trusting it doubled the 11008x4096 time).
template <int FMT, int NB>
TcPlan tc_plan_t(const vxb_ctx *ctx, const TiledGeom &g) {
  using SM = TcSmem<FMT, NB>;
  const int sms = ctx->num_sms > 0 ? ctx->num_sms : 148;
  const int n_wst = g.n_chunks / TcGeo<FMT>::CPS;
  TcPlan best;
  double best_cost = 1e30;
  for (int S = 1; S <= 8; S++) {
    if (S > n_wst) break;
    const int ctas = g.n_groups * S;
    const int per_cta = (n_wst + S - 1) / S;
    int wr = TC_MAX_WR;
    while (wr > 2 && SM::bytes(wr) > TC_SMEM_CAP) wr--;
    wr = std::min(wr, std::max(per_cta, 1));
    const size_t smem = SM::bytes(wr);
    // CTAs per SM: the shared memory allows two (the 1-KB per-CTA reserve
    // included) and the registers are bounded for two by __launch_bounds__
    const int per_sm = std::min<int>(2, (int)(((size_t)228 << 10) / (smem + 1024)));
    if (per_sm < 1 || tc_resident<FMT, NB>(smem, 1, sms) < 1) continue;
    const int slots = per_sm * sms;
    const int waves = (ctas + slots - 1) / slots;
    if (waves > 1 && S > 1) continue;  // a split that needs a second wave never pays
    // clusters pack into the GPCs with some loss: a cluster split must leave a
    // tenth of the slots free to stay in one wave
    if (S > 1 && ctas * 10 > slots * 9) continue;
    // stages of the busiest SM: its CTAs (one wave at a time) share it
    const int on_sm = std::min(per_sm, (std::min(ctas, slots) + sms - 1) / sms);
    const double t_stage = on_sm > 1 ? 0.55 : 1.0;  // per CTA and stage, relative: two CTAs overlap
    const double cost = (double)waves * per_cta * on_sm * t_stage + (S > 1 ? 0.7 : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best.S = S;
      best.wr = wr;
      best.n_wst = n_wst;
      best.smem = smem;
    }
  }
  return best;
}

// The tiled units as a 3-D u32 tensor [tiles][chunks][unit words]: boxes of
// 8 tiles x cps chunks x one unit (one stage).
int weights_tensor_map(vxb_ctx *ctx, const uint8_t *units, const TiledGeom &g, int cps, CUtensorMap *map) {
  const EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return set_error(ctx, VXB_ECUDA, "vxb_gemv_q: cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {(cuuint64_t)(g.unit / 4), (cuuint64_t)g.n_chunks, (cuuint64_t)g.n_tiles};
  cuuint64_t strides[2] = {(cuuint64_t)g.unit, (cuuint64_t)g.n_chunks * g.unit};
  cuuint32_t box[3] = {(cuuint32_t)(g.unit / 4), (cuuint32_t)cps, 8};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t *>(units), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: weight tensor map failed (%d)", (int)r);
  return VXB_OK;
}

// x bf16 [B, K] as boxes of 64 columns x NB rows with the 128-byte swizzle
// (rows past B and columns past K read as zeros)
int x_tensor_map_rows(vxb_ctx *ctx, const uint16_t *x, int B, int K, int NB, CUtensorMap *map) {
  const EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return set_error(ctx, VXB_ECUDA, "vxb_gemv_q: cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)B};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)NB};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: activation tensor map failed (%d)", (int)r);
  return VXB_OK;
}

template <int FMT, int NB>
int tc_launch_t(vxb_ctx *ctx, const TcArgs &a0, const uint16_t *x, const TiledGeom &g, cudaStream_t st, bool pdl) {
  auto kfn = gemv_tc_kernel<FMT, NB>;
  const TcPlan p = tc_plan_t<FMT, NB>(ctx, g);
  if (p.S == 0) return set_error(ctx, VXB_EINVAL, "vxb_gemv_q: no tensor-core launch plan fits N=%d K=%d", a0.N, a0.K);
  CUtensorMap wmap, xmap;
  if (int rc = weights_tensor_map(ctx, a0.units, g, TcGeo<FMT>::CPS, &wmap)) return rc;
  if (int rc = x_tensor_map_rows(ctx, x, a0.B, a0.K, NB, &xmap)) return rc;
  static std::atomic<bool> configured[64];  // kernel attributes set on this device (zero-initialized)
  const int dev = ctx->device & 63;
  if (!configured[dev]) {
    VXB_CUDA_TRY(ctx, cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM_CAP));
    configured[dev] = true;
  }
  TcArgs a = a0;
  a.wr = p.wr;
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
  VXB_CUDA_TRY(ctx, cudaLaunchKernelEx(&cfg, kfn, wmap, xmap, a));
  return VXB_OK;
}

// Routing by measurement (kernel_bench, back-to-back launches over rotating
// weight copies): the tensor-core kernel is faster than the mma.sync group
// kernel on up to 16k rows for Q4_0 from batch 17 and for Q8_0 from batch 9
// (batch 32, Q4_0: 4096x4096 10.0 us against 11.8, 4096x11008 18.6 against
// 21.9, 11008x4096 19.6 against 22.0, 12288x4096 25.8 against 31.4), and on
// more rows at batch 28 and above (22016x4096 41.2 against 43.8, 32000x4096
// 41.9 against 50.5); Q8_0 with 28k rows and more takes it at every batch
// (32000x4096, batch 9: 45.7 against 49.5).
// VXB_GEMV_TCGEN05=1 sends every batch 9-32 to it, =0 none.
int tc_mode() {
  static const int mode = [] {
    const char *v = getenv("VXB_GEMV_TCGEN05");
    if (v && v[0] == '1') return 1;
    if (v && v[0] == '0') return 0;
    return -1;
  }();
  return mode;
}

}  // namespace

namespace vxb {

// y = W x (+ resid) for batches 9..32 through the tcgen05 kernel.
int gemv_tc(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, const uint16_t *d_x, int batch, int y_dtype,
            void *d_y, const float *d_resid, int *d_err, cudaStream_t st, bool pdl) {
  const TiledGeom g = tiled_geom(fmt, N, K);
  TcArgs a = {};
  const uint8_t *base = (const uint8_t *)d_tiled;
  a.units = base + g.codes_off;
  a.hdr = (const uint32_t *)base;
  a.y = d_y;
  a.resid = d_resid;
  a.err = d_err;
  a.N = N;
  a.K = K;
  a.B = batch;
  a.n_chunks = g.n_chunks;
  a.y_dtype = y_dtype;
  if (fmt == VXB_Q4_0)
    return batch <= 16 ? tc_launch_t<0, 16>(ctx, a, d_x, g, st, pdl) : tc_launch_t<0, 32>(ctx, a, d_x, g, st, pdl);
  return batch <= 16 ? tc_launch_t<1, 16>(ctx, a, d_x, g, st, pdl) : tc_launch_t<1, 32>(ctx, a, d_x, g, st, pdl);
}

bool gemv_tc_eligible(int fmt, int N, int batch) {
  if (batch < 9 || batch > 32) return false;
  const int m = tc_mode();
  if (m >= 0) return m == 1;
  // up to 16k rows the row groups' k-splits fill one wave of two CTAs per SM
  if (N <= 16384) return fmt == VXB_Q8_0 || batch >= 17;
  if (fmt == VXB_Q8_0 && N >= 28000) return true;
  return N >= 16384 && batch >= 28;
}

int gemv_tc_splits(const vxb_ctx *ctx, int fmt, int N, int K, int batch) {
  const TiledGeom g = tiled_geom(fmt, N, K);
  if (fmt == VXB_Q4_0) return batch <= 16 ? tc_plan_t<0, 16>(ctx, g).S : tc_plan_t<0, 32>(ctx, g).S;
  return batch <= 16 ? tc_plan_t<1, 16>(ctx, g).S : tc_plan_t<1, 32>(ctx, g).S;
}

}  // namespace vxb
