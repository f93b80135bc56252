// Internal interface of the tensor-parallel communicator (comm.cu).
#pragma once

#include "vxb_internal.h"

// One-shot all-reduce over NVLink peer memory for decode-sized messages (up
// to kArOneShotBytes of f32): every rank's buffer is mapped into every other
// rank with CUDA IPC. A buffer holds, for each of three generations, one slot
// per source rank (filled with the empty marker between uses), then the
// per-block generation counters.
constexpr int kArMaxRanks = 8;
constexpr int kArBlocks = 32;  // CTAs (message slices) per call
constexpr int kArGens = 3;     // generations rotating through the slots
// messages up to this size take the one-shot path (NCCL above)
constexpr size_t kArOneShotBytes = (size_t)512 << 10;
constexpr size_t kArSlotBytes = kArOneShotBytes;  // per (generation, source rank)
constexpr size_t kArCountersOff = (size_t)kArGens * kArMaxRanks * kArSlotBytes;
constexpr size_t kArBytes = kArCountersOff + (size_t)kArBlocks * 4;
constexpr uint32_t kArEmpty = 0xFFFFFFFFu;  // a NaN bit pattern no sent value has

struct vxb_comm {
  vxb_ctx *ctx = nullptr;
  void *nccl = nullptr;  // ncclComm_t
  int nranks = 1, rank = 0;
  uint8_t *ar_local = nullptr;                  // this rank's buffer (cudaMalloc)
  uint8_t *ar_peer[kArMaxRanks] = {nullptr};    // every rank's buffer (own one included)
  bool ar_ready = false;
};

namespace vxb {

#ifdef __CUDACC__
__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const void *p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Poll a 16-byte peer slot until none of its words holds the empty marker;
// false (with whatever the slot held last in *out) once `budget` SM clock
// cycles have passed.
__device__ __forceinline__ bool wait_slot_filled(const void *slot, uint4 *out, long long budget) {
  uint4 v = ld_relaxed_sys_v4(slot);
  const long long t0 = clock64();
  while (v.x == kArEmpty || v.y == kArEmpty || v.z == kArEmpty || v.w == kArEmpty) {
    if (clock64() - t0 > budget) {
      *out = v;
      return false;
    }
    v = ld_relaxed_sys_v4(slot);
  }
  *out = v;
  return true;
}
#endif

// op 0 = sum, 1 = max; dtype VXB_F32, VXB_BF16 or -1 for u64 (max of packed keys)
int comm_allreduce(vxb_comm *c, void *buf, size_t count, int dtype, int op, cudaStream_t st);
int comm_allgather_f32(vxb_comm *c, const float *send, float *recv, size_t count, cudaStream_t st);

}  // namespace vxb
