// Tensor-parallel communicator: NCCL over NVLink / NVSwitch, opened at run
// time (dlopen of libnccl.so.2, so the library carries no link-time NCCL
// dependency and shares the process's NCCL when one is already loaded).
//
// Replaces the nccl_ffi.rs externs (src/nccl_ffi.rs:12-72): a unique id is
// created on one rank, shared by the caller's own channel (a store, MPI, a
// file), and every rank joins with vxb_comm_init. Collectives run on the
// caller's stream and may be captured into CUDA graphs.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "comm.h"

using namespace vxb;

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
  char why[256] = {0};
};

NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      snprintf(api.why, sizeof(api.why), "cannot open libnccl.so.2: %s", dlerror());
      return;
    }
    api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
    api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
    api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
    api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
    api.all_gather = (decltype(api.all_gather))dlsym(h, "ncclAllGather");
    api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.all_gather &&
             api.error_string;
    if (!api.ok) snprintf(api.why, sizeof(api.why), "libnccl.so.2 lacks an entry point");
  });
  return api;
}

int nccl_fail(vxb_ctx *ctx, ncclResult_t r, const char *what) {
  return set_error(ctx, VXB_ENCCL, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

}  // namespace

namespace vxb {

int comm_allreduce(vxb_comm *c, void *buf, size_t count, int dtype, int op, cudaStream_t st) {
  NcclApi &n = nccl();
  const ncclDataType_t t = dtype == VXB_F32 ? ncclFloat32 : dtype == VXB_BF16 ? ncclBfloat16 : ncclUint64;
  const ncclRedOp_t o = op == 0 ? ncclSum : ncclMax;
  const ncclResult_t r = n.all_reduce(buf, buf, count, t, o, (ncclComm_t)c->nccl, st);
  if (r != ncclSuccess) return nccl_fail(c->ctx, r, "ncclAllReduce");
  return VXB_OK;
}

int comm_allgather_f32(vxb_comm *c, const float *send, float *recv, size_t count, cudaStream_t st) {
  const ncclResult_t r = nccl().all_gather(send, recv, count, ncclFloat32, (ncclComm_t)c->nccl, st);
  if (r != ncclSuccess) return nccl_fail(c->ctx, r, "ncclAllGather");
  return VXB_OK;
}

}  // namespace vxb

VXB_API int vxb_nccl_unique_id(void *h_out) {
  if (!h_out) return set_error(nullptr, VXB_EINVAL, "vxb_nccl_unique_id: null output");
  NcclApi &n = nccl();
  if (!n.ok) return set_error(nullptr, VXB_ENCCL, "vxb_nccl_unique_id: %s", n.why);
  ncclUniqueId id;
  const ncclResult_t r = n.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(nullptr, r, "ncclGetUniqueId");
  memcpy(h_out, id.internal, NCCL_UNIQUE_ID_BYTES);
  return VXB_OK;
}

VXB_API int vxb_comm_init(vxb_ctx *ctx, int nranks, int rank, const void *h_unique_id, vxb_comm **out) {
  if (!ctx || !h_unique_id || !out) return set_error(ctx, VXB_EINVAL, "vxb_comm_init: null argument");
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return set_error(ctx, VXB_EINVAL, "vxb_comm_init: rank %d of %d", rank, nranks);
  NcclApi &n = nccl();
  if (!n.ok) return set_error(ctx, VXB_ENCCL, "vxb_comm_init: %s", n.why);
  if (int rc = use_device(ctx)) return rc;
  ncclUniqueId id;
  memcpy(id.internal, h_unique_id, NCCL_UNIQUE_ID_BYTES);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = n.comm_init_rank(&comm, nranks, id, rank);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclCommInitRank");
  vxb_comm *c = new vxb_comm();
  c->ctx = ctx;
  c->nccl = comm;
  c->nranks = nranks;
  c->rank = rank;
  *out = c;
  return VXB_OK;
}

VXB_API int vxb_comm_destroy(vxb_comm *c) {
  if (!c) return VXB_OK;
  if (c->nccl) nccl().comm_destroy((ncclComm_t)c->nccl);
  delete c;
  return VXB_OK;
}

VXB_API int vxb_allreduce_sum(vxb_comm *c, void *d_buf, size_t count, int dtype, void *stream) {
  if (!c || !d_buf) return set_error(c ? c->ctx : nullptr, VXB_EINVAL, "vxb_allreduce_sum: null argument");
  if (dtype != VXB_F32 && dtype != VXB_BF16) return set_error(c->ctx, VXB_EINVAL, "vxb_allreduce_sum: dtype");
  if (int rc = use_device(c->ctx)) return rc;
  return comm_allreduce(c, d_buf, count, dtype, 0, (cudaStream_t)stream);
}
