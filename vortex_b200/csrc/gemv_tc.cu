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

// Bounded wait by all lanes of a warp with a warp-uniform outcome (the lanes
// stay converged for the elected arrivals); a failure is recorded once and
// later waits are skipped.
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
  static std::atomic<bool> configured[64];  // kernel attributes set on this device (zero-initialized)
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

bool gemv_tc_eligible(int batch) { return tc_enabled() && batch >= 9 && batch <= 32; }

}  // namespace vxb
