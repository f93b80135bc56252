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
#include <vector>

#include "comm.h"
#include "tc_common.h"

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

// ---------------------------------------------------------------------------
// One-shot all-reduce (sum, f32) over peer memory without flags: the arrival
// of the data is the signal. Every slot of a buffer holds the empty marker
// (0xFFFFFFFF) between uses. CTA b owns slice b of the message: it stores its
// slice of the input (NaNs made canonical, so no value equals the marker)
// into slot (generation g mod 3, this rank) of every rank's buffer with
// relaxed system-scope stores, then polls the slots (g mod 3, 0..nranks-1) of
// its own buffer until no element holds the marker (bounded), sums them in
// rank order - the same order on every rank, so all ranks hold identical bits
// - and writes the marker back. A rank can run at most one call ahead of the
// slowest rank (it needs everybody's data to finish a call), so with three
// generations a slot is written again only after its reader has emptied it.
// The generation of block b is a per-block device counter (the same sequence
// of calls on every rank, CUDA graphs included). No fences on the path: one
// NVLink write latency per call.
struct ArArgs {
  uint8_t *peer[kArMaxRanks];
  float *data;  // in / out (in place)
  int *err;
  size_t n;
  int rank, nranks;
};

__device__ __forceinline__ void st_relaxed_sys_v4(void *p, uint4 v) {
  asm volatile("st.relaxed.sys.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint32_t canon_bits(float f) { return f != f ? 0x7FC00000u : __float_as_uint(f); }

__global__ void __launch_bounds__(512) oneshot_allreduce_kernel(const ArArgs a) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.x;
  __shared__ uint32_t s_gen;
  __shared__ uint8_t *s_peer[kArMaxRanks];  // indexed by rank below (no local-memory copy of the argument)
  if (threadIdx.x == 0) {
#pragma unroll
    for (int q = 0; q < kArMaxRanks; q++) s_peer[q] = a.peer[q];
  }
  __syncthreads();
  uint8_t *mine = s_peer[a.rank];
  uint32_t *counter = reinterpret_cast<uint32_t *>(mine + kArCountersOff) + b;
  if (threadIdx.x == 0) s_gen = __ldcg(counter) + 1;
  __syncthreads();
  const uint32_t gen = s_gen;
  const size_t gbase = (size_t)(gen % kArGens) * kArMaxRanks * kArSlotBytes;
  // slice of this block, in 16-byte units (the message is padded to them)
  const size_t n4 = (a.n + 3) / 4;
  const size_t per = (n4 + kArBlocks - 1) / kArBlocks;
  const size_t i0 = (size_t)b * per, i1 = min(n4, i0 + per);
  for (size_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const size_t e = i * 4;
    uint4 v;
    v.x = canon_bits(e < a.n ? __ldcg(a.data + e) : 0.f);
    v.y = canon_bits(e + 1 < a.n ? __ldcg(a.data + e + 1) : 0.f);
    v.z = canon_bits(e + 2 < a.n ? __ldcg(a.data + e + 2) : 0.f);
    v.w = canon_bits(e + 3 < a.n ? __ldcg(a.data + e + 3) : 0.f);
    for (int q = 0; q < a.nranks; q++)
      st_relaxed_sys_v4(s_peer[q] + gbase + (size_t)a.rank * kArSlotBytes + i * 16, v);
  }
  for (size_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < a.nranks; q++) {
      uint8_t *slot = mine + gbase + (size_t)q * kArSlotBytes + i * 16;
      uint4 v;
      if (!wait_slot_filled(slot, &v, vxb::tc::kWaitBudget)) atomicExch(a.err, 1);
      acc.x += __uint_as_float(v.x);
      acc.y += __uint_as_float(v.y);
      acc.z += __uint_as_float(v.z);
      acc.w += __uint_as_float(v.w);
      st_relaxed_sys_v4(slot, make_uint4(kArEmpty, kArEmpty, kArEmpty, kArEmpty));
    }
    const size_t e = i * 4;
    if (e < a.n) a.data[e] = acc.x;
    if (e + 1 < a.n) a.data[e + 1] = acc.y;
    if (e + 2 < a.n) a.data[e + 2] = acc.z;
    if (e + 3 < a.n) a.data[e + 3] = acc.w;
  }
  __syncthreads();
  if (threadIdx.x == 0) *counter = gen;
}

// Collective set-up of the peer buffers: allocate, zero, exchange IPC handles
// through NCCL, open every peer's buffer.
int ar_setup(vxb_comm *c) {
  if (c->nranks < 2 || c->nranks > kArMaxRanks) return VXB_OK;  // NCCL only
  vxb_ctx *ctx = c->ctx;
  if (cudaMalloc(&c->ar_local, kArBytes) != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, VXB_ENOMEM, "vxb_comm_init: peer buffer");
  }
  VXB_CUDA_TRY(ctx, cudaMemset(c->ar_local, 0xFF, kArCountersOff));  // every slot empty
  VXB_CUDA_TRY(ctx, cudaMemset(c->ar_local + kArCountersOff, 0, kArBytes - kArCountersOff));
  cudaIpcMemHandle_t h;
  VXB_CUDA_TRY(ctx, cudaIpcGetMemHandle(&h, c->ar_local));
  uint8_t *d_handles = nullptr;
  VXB_CUDA_TRY(ctx, cudaMalloc(&d_handles, sizeof(h) * (c->nranks + 1)));
  VXB_CUDA_TRY(ctx, cudaMemcpy(d_handles + sizeof(h) * c->nranks, &h, sizeof(h), cudaMemcpyHostToDevice));
  VXB_CUDA_TRY(ctx, cudaDeviceSynchronize());
  const ncclResult_t r = nccl().all_gather(d_handles + sizeof(h) * c->nranks, d_handles, sizeof(h), ncclUint8,
                                           (ncclComm_t)c->nccl, 0);
  std::vector<cudaIpcMemHandle_t> all(c->nranks);
  cudaError_t e = cudaStreamSynchronize(0);
  if (e == cudaSuccess) e = cudaMemcpy(all.data(), d_handles, sizeof(h) * c->nranks, cudaMemcpyDeviceToHost);
  cudaFree(d_handles);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclAllGather of IPC handles");
  if (e != cudaSuccess) return cuda_fail(ctx, e, "IPC handle exchange");
  for (int q = 0; q < c->nranks; q++) {
    if (q == c->rank) {
      c->ar_peer[q] = c->ar_local;
      continue;
    }
    void *p = nullptr;
    e = cudaIpcOpenMemHandle(&p, all[q], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaIpcOpenMemHandle");
    c->ar_peer[q] = (uint8_t *)p;
  }
  c->ar_ready = true;
  return VXB_OK;
}

}  // namespace

namespace vxb {

int comm_allreduce(vxb_comm *c, void *buf, size_t count, int dtype, int op, cudaStream_t st) {
  if (c->ar_ready && dtype == VXB_F32 && op == 0 && count > 0 && (count + 3) / 4 * 16 <= kArOneShotBytes) {
    if (int rc = ws_reserve(c->ctx, 0, 0)) return rc;  // device error word
    ArArgs a;
    for (int q = 0; q < kArMaxRanks; q++) a.peer[q] = c->ar_peer[q];
    a.data = (float *)buf;
    a.err = c->ctx->d_err;
    a.n = count;
    a.rank = c->rank;
    a.nranks = c->nranks;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kArBlocks);
    cfg.blockDim = dim3(512);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VXB_CUDA_TRY(c->ctx, cudaLaunchKernelEx(&cfg, oneshot_allreduce_kernel, a));
    return VXB_OK;
  }
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
  if (int rc = ar_setup(c)) {
    vxb_comm_destroy(c);
    return rc;
  }
  *out = c;
  return VXB_OK;
}

// Collective: every rank calls it. A barrier (NCCL all-reduce) first, so no
// rank frees its peer buffer while another rank may still read it.
VXB_API int vxb_comm_destroy(vxb_comm *c) {
  if (!c) return VXB_OK;
  use_device(c->ctx);
  cudaDeviceSynchronize();
  if (c->nccl && c->ar_ready) {
    float *one = nullptr;
    if (cudaMalloc(&one, sizeof(float)) == cudaSuccess) {
      nccl().all_reduce(one, one, 1, ncclFloat32, ncclSum, (ncclComm_t)c->nccl, 0);
      cudaStreamSynchronize(0);
      cudaFree(one);
    }
    cudaGetLastError();
  }
  for (int q = 0; q < kArMaxRanks; q++)
    if (c->ar_peer[q] && q != c->rank) cudaIpcCloseMemHandle(c->ar_peer[q]);
  if (c->ar_local) cudaFree(c->ar_local);
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
