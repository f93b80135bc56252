// Internal interface of the tensor-parallel communicator (comm.cu).
#pragma once

#include "vxb_internal.h"

// One-shot all-reduce over NVLink peer memory for decode-sized messages
// (up to kArMaxBytes of f32): every rank's buffer is mapped into every other
// rank with CUDA IPC.
constexpr int kArMaxRanks = 8;
constexpr int kArBlocks = 32;                      // CTAs (message slices) per call
constexpr size_t kArMaxBytes = (size_t)1 << 20;    // per slot
// messages up to this size take the one-shot path (measured on 8 B200s: 18-36
// us against NCCL's 36-40 us up to 512 KiB; NCCL wins from about 1 MiB)
constexpr size_t kArOneShotBytes = (size_t)512 << 10;
constexpr size_t kArFlagsOff = 2 * kArMaxBytes;    // two data slots, then flags
constexpr size_t kArBytes = kArFlagsOff + (size_t)kArBlocks * kArMaxRanks * 4 + (size_t)kArBlocks * 4;

struct vxb_comm {
  vxb_ctx *ctx = nullptr;
  void *nccl = nullptr;  // ncclComm_t
  int nranks = 1, rank = 0;
  uint8_t *ar_local = nullptr;                  // this rank's buffer (cudaMalloc)
  uint8_t *ar_peer[kArMaxRanks] = {nullptr};    // every rank's buffer (own one included)
  bool ar_ready = false;
};

namespace vxb {

// op 0 = sum, 1 = max; dtype VXB_F32, VXB_BF16 or -1 for u64 (max of packed keys)
int comm_allreduce(vxb_comm *c, void *buf, size_t count, int dtype, int op, cudaStream_t st);
int comm_allgather_f32(vxb_comm *c, const float *send, float *recv, size_t count, cudaStream_t st);

}  // namespace vxb
