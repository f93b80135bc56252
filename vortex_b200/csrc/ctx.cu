// Context, errors and memory entry points of the C ABI.
// Replaces gpu_runtime::CpuRuntime allocation/copy (src/gpu_runtime.rs:297-348).
#include "gemv.h"
#include "vxb_internal.h"

namespace vxb {

static std::mutex g_err_mu;
static std::string g_err;

int set_error(vxb_ctx *ctx, int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (ctx) {
    ctx->err = buf;
  } else {
    std::lock_guard<std::mutex> g(g_err_mu);
    g_err = buf;
  }
  return code;
}

int cuda_fail(vxb_ctx *ctx, cudaError_t e, const char *what) {
  return set_error(ctx, VXB_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int use_device(vxb_ctx *ctx) {
  int cur = -1;
  VXB_CUDA_TRY(ctx, cudaGetDevice(&cur));
  if (cur != ctx->device) VXB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
  return VXB_OK;
}

int ws_reserve(vxb_ctx *ctx, size_t bytes, size_t counters) {
  if (!ctx->d_err) {
    int *p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) {
      cudaGetLastError();
      return set_error(ctx, VXB_ENOMEM, "device error word allocation failed");
    }
    VXB_CUDA_TRY(ctx, cudaMemset(p, 0, sizeof(int)));
    ctx->d_err = p;
  }
  if (bytes > ctx->ws_bytes) {
    size_t nb = round_up(bytes > (size_t)16 << 20 ? bytes : (size_t)16 << 20, 1 << 20);
    void *p = nullptr;
    // work already queued may still read the old buffer
    if (ctx->ws) {
      VXB_CUDA_TRY(ctx, cudaDeviceSynchronize());
      VXB_CUDA_TRY(ctx, cudaFree(ctx->ws));
    }
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
    if (cudaMalloc(&p, nb) != cudaSuccess) {
      cudaGetLastError();
      return set_error(ctx, VXB_ENOMEM, "workspace allocation of %zu bytes failed", nb);
    }
    ctx->ws = p;
    ctx->ws_bytes = nb;
  }
  if (counters > ctx->n_counters) {
    size_t nc = round_up(counters > 4096 ? counters : 4096, 1024);
    unsigned *p = nullptr;
    if (ctx->counters) {
      VXB_CUDA_TRY(ctx, cudaDeviceSynchronize());
      VXB_CUDA_TRY(ctx, cudaFree(ctx->counters));
    }
    ctx->counters = nullptr;
    ctx->n_counters = 0;
    if (cudaMalloc(&p, nc * sizeof(unsigned)) != cudaSuccess) {
      cudaGetLastError();
      return set_error(ctx, VXB_ENOMEM, "counter allocation failed");
    }
    VXB_CUDA_TRY(ctx, cudaMemset(p, 0, nc * sizeof(unsigned)));
    ctx->counters = p;
    ctx->n_counters = nc;
  }
  return VXB_OK;
}

}  // namespace vxb

using namespace vxb;

VXB_API int vxb_abi_version(void) { return VXB_ABI_VERSION; }

VXB_API int vxb_device_count(int *count) {
  if (!count) return set_error(nullptr, VXB_EINVAL, "vxb_device_count: null output");
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    cudaGetLastError();
    return cuda_fail(nullptr, e, "cudaGetDeviceCount");
  }
  return VXB_OK;
}

VXB_API int vxb_init(int device, vxb_ctx **out) {
  if (!out) return set_error(nullptr, VXB_EINVAL, "vxb_init: null output");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceCount");
  if (device < 0 || device >= n)
    return set_error(nullptr, VXB_EINVAL, "vxb_init: device %d out of range (%d devices)", device, n);
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaSetDevice");
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceProperties");
  if (prop.major != 10)
    return set_error(nullptr, VXB_EUNSUPPORTED,
                     "vxb_init: device %d is sm_%d%d; the library is compiled for sm_100a (B200)", device,
                     prop.major, prop.minor);
  vxb_ctx *ctx = new vxb_ctx();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  ctx->smem_optin = prop.sharedMemPerBlockOptin;
  *out = ctx;
  return VXB_OK;
}

VXB_API int vxb_destroy(vxb_ctx *ctx) {
  if (!ctx) return VXB_OK;
  int cur = -1;
  cudaGetDevice(&cur);
  cudaSetDevice(ctx->device);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->counters) cudaFree(ctx->counters);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->gemm_ws) cudaFree(ctx->gemm_ws);
  if (cur >= 0) cudaSetDevice(cur);
  delete ctx;
  return VXB_OK;
}

VXB_API const char *vxb_last_error(const vxb_ctx *ctx) {
  if (ctx) return ctx->err.c_str();
  std::lock_guard<std::mutex> g(g_err_mu);
  return g_err.c_str();
}

VXB_API int vxb_alloc(vxb_ctx *ctx, size_t bytes, void **d_out) {
  if (!ctx || !d_out) return set_error(ctx, VXB_EINVAL, "vxb_alloc: null argument");
  int rc = use_device(ctx);
  if (rc) return rc;
  *d_out = nullptr;
  if (bytes == 0) return VXB_OK;
  if (cudaMalloc(d_out, bytes) != cudaSuccess) {
    cudaGetLastError();
    *d_out = nullptr;
    return set_error(ctx, VXB_ENOMEM, "vxb_alloc: %zu bytes failed", bytes);
  }
  return VXB_OK;
}

VXB_API int vxb_free(vxb_ctx *ctx, void *d_ptr) {
  if (!ctx) return set_error(ctx, VXB_EINVAL, "vxb_free: null context");
  if (!d_ptr) return VXB_OK;
  int rc = use_device(ctx);
  if (rc) return rc;
  VXB_CUDA_TRY(ctx, cudaFree(d_ptr));
  return VXB_OK;
}

VXB_API int vxb_memcpy_h2d(vxb_ctx *ctx, void *d_dst, const void *h_src, size_t bytes, void *stream) {
  if (!ctx || (bytes && (!d_dst || !h_src))) return set_error(ctx, VXB_EINVAL, "vxb_memcpy_h2d: null argument");
  int rc = use_device(ctx);
  if (rc) return rc;
  VXB_CUDA_TRY(ctx, cudaMemcpyAsync(d_dst, h_src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream));
  return VXB_OK;
}

VXB_API int vxb_memcpy_d2h(vxb_ctx *ctx, void *h_dst, const void *d_src, size_t bytes, void *stream) {
  if (!ctx || (bytes && (!h_dst || !d_src))) return set_error(ctx, VXB_EINVAL, "vxb_memcpy_d2h: null argument");
  int rc = use_device(ctx);
  if (rc) return rc;
  VXB_CUDA_TRY(ctx, cudaMemcpyAsync(h_dst, d_src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  VXB_CUDA_TRY(ctx, cudaStreamSynchronize((cudaStream_t)stream));
  return VXB_OK;
}

VXB_API int vxb_memset(vxb_ctx *ctx, void *d_dst, int value, size_t bytes, void *stream) {
  if (!ctx || (bytes && !d_dst)) return set_error(ctx, VXB_EINVAL, "vxb_memset: null argument");
  int rc = use_device(ctx);
  if (rc) return rc;
  VXB_CUDA_TRY(ctx, cudaMemsetAsync(d_dst, value, bytes, (cudaStream_t)stream));
  return VXB_OK;
}

// Two words can hold a timeout: the context's own (allocated with its
// workspace) and the one in vxb_gemv_q_static's fixed array on this device
// (shared by every context of the device, so reading it here clears it for
// all of them). Neither read nor clear allocates.
VXB_API int vxb_device_error(vxb_ctx *ctx, int *out) {
  if (!ctx || !out) return set_error(ctx, VXB_EINVAL, "vxb_device_error: null argument");
  *out = 0;
  int *words[2] = {ctx->d_err, static_error_word(ctx->device)};
  if (!words[0] && !words[1]) return VXB_OK;
  if (int rc = use_device(ctx)) return rc;
  VXB_CUDA_TRY(ctx, cudaDeviceSynchronize());
  for (int *w : words) {
    if (!w) continue;
    int v = 0;
    VXB_CUDA_TRY(ctx, cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
    if (v) VXB_CUDA_TRY(ctx, cudaMemset(w, 0, sizeof(int)));
    if (v && !*out) *out = v;
  }
  if (*out) return set_error(ctx, VXB_ETIMEOUT, "a bounded device wait timed out (error word %d)", *out);
  return VXB_OK;
}

VXB_API int vxb_sync(vxb_ctx *ctx, void *stream) {
  if (!ctx) return set_error(ctx, VXB_EINVAL, "vxb_sync: null context");
  int rc = use_device(ctx);
  if (rc) return rc;
  VXB_CUDA_TRY(ctx, cudaStreamSynchronize((cudaStream_t)stream));
  return VXB_OK;
}
