// Internal interface of the tensor-parallel communicator (comm.cu).
#pragma once

#include "vxb_internal.h"

struct vxb_comm {
  vxb_ctx *ctx = nullptr;
  void *nccl = nullptr;  // ncclComm_t
  int nranks = 1, rank = 0;
};

namespace vxb {

// op 0 = sum, 1 = max; dtype VXB_F32, VXB_BF16 or -1 for u64 (max of packed keys)
int comm_allreduce(vxb_comm *c, void *buf, size_t count, int dtype, int op, cudaStream_t st);
int comm_allgather_f32(vxb_comm *c, const float *send, float *recv, size_t count, cudaStream_t st);

}  // namespace vxb
