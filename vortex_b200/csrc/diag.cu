// Self-test of the bounded device-side waits.
//
// Every wait in the library's kernels - the mbarrier phases of the K1-K4
// stage rings and the peer-slot polls of the one-shot all-reduce - gives up
// after a cycle budget, sets a device error word and lets the kernel finish,
// so a producer that never arrives (a lost copy, a rank that died) ends in
// VXB_ETIMEOUT from vxb_device_error instead of a hung GPU. This entry point
// runs those same wait helpers on something nothing will ever complete (an
// mbarrier nobody arrives on, a slot holding the empty marker) with a short
// budget, so the timeout path can be exercised on a healthy device.
#include "comm.h"
#include "gemv.h"
#include "tc_common.h"
#include "vxb_internal.h"

using namespace vxb;

namespace {

__global__ void wait_selftest_kernel(int kind, const void *slot, long long budget, int *err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  if (kind == 0) {
    tc::mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc::wait_or_flag(&bar, 0, err, budget);  // nobody arrives
  } else {
    uint4 v;
    if (!wait_slot_filled(slot, &v, budget)) atomicExch(err, 1);  // nobody writes the slot
  }
}

}  // namespace

VXB_API int vxb_selftest_wait_timeout(vxb_ctx *ctx, int kind, int static_word, long long budget_cycles,
                                      void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_selftest_wait_timeout: null context");
  if (kind != 0 && kind != 1) return set_error(ctx, VXB_EINVAL, "vxb_selftest_wait_timeout: kind %d", kind);
  if (budget_cycles < 1 || budget_cycles > tc::kWaitBudget)
    return set_error(ctx, VXB_EINVAL, "vxb_selftest_wait_timeout: budget %lld outside 1..2^31", budget_cycles);
  if (int rc = use_device(ctx)) return rc;
  // the slot lives in the context workspace (16 bytes of the empty marker)
  if (int rc = ws_reserve(ctx, 256, 0)) return rc;
  int *err = ctx->d_err;
  if (static_word)
    if (int rc = static_error_word_resolve(ctx, &err)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  VXB_CUDA_TRY(ctx, cudaMemsetAsync(ctx->ws, 0xFF, 16, st));
  wait_selftest_kernel<<<1, 32, 0, st>>>(kind, ctx->ws, budget_cycles, err);
  return launch_check(ctx, "wait_selftest_kernel");
}
