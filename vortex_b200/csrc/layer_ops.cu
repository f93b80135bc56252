// K5: the small per-token kernels of the Llama-style decoder block
// (stdlib/ai/transformer.vx:413-603):
//   rmsnorm_bias : x * w / sqrt(mean(x^2) + eps) + b            (413-439)
//   rope         : adjacent pairs (x[2i], x[2i+1]) of the whole projection
//                  rotated by theta = pos / exp(i * ln(10000) / dim) (442-466)
//   swiglu       : silu(W1 x) * (W3 x), silu(x) = x * sigmoid(x)   (591-603, 176-182)
//   embed        : token embedding row -> f32 residual stream
//   argmax       : greedy next token, first index of the maximum (1163-1177)
// Accumulation is f32; the GEMV inputs are rounded once to bf16.
#include <cuda_bf16.h>

#include "layer_ops.h"

using namespace vxb;

namespace {

__device__ __forceinline__ float block_sum(float v, float *red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

__global__ void rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ b,
                               int n, float eps, uint16_t *__restrict__ out) {
  __shared__ float red[32];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const float *xr = x + (size_t)blockIdx.x * n;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)n + eps);
  uint16_t *o = out + (size_t)blockIdx.x * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = f32_to_bf16_bits(xr[i] * inv * w[i] + b[i]);
}

// qkv: f32 [B, dim + 2*kvdim] (q | k | v); positions from the KV placements
// of layer 0 of this step. Writes q (bf16 [B, dim]), the new keys at
// k_out [B, kvdim] and the new values at v_out [B, kvdim] (bf16).
// q_pair0 / k_pair0: index of the first rotation pair of this q / k slice in
// the full vectors (tensor-parallel shards hold a slice of the heads)
__global__ void rope_kernel(const float *__restrict__ qkv, int dim, int kvdim, const KVPlace *__restrict__ places,
                            const double *__restrict__ rope_div, uint16_t *__restrict__ q_out,
                            uint16_t *__restrict__ k_out, uint16_t *__restrict__ v_out, int q_pair0, int k_pair0) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const int b = blockIdx.x;
  const double pos = (double)places[b].pos;
  const float *row = qkv + (size_t)b * (dim + 2 * kvdim);
  uint16_t *qo = q_out + (size_t)b * dim;
  uint16_t *ko = k_out + (size_t)b * kvdim;
  uint16_t *vo = v_out + (size_t)b * kvdim;
  const int npq = dim / 2, npk = kvdim / 2;
  for (int p = threadIdx.x; p < npq + npk; p += blockDim.x) {
    const bool isk = p >= npq;
    const int pi = isk ? p - npq : p;
    // theta in f64 (pos / divisor), then sin/cos
    double s, c;
    sincos(pos / rope_div[pi + (isk ? k_pair0 : q_pair0)], &s, &c);
    const float cf = (float)c, sf = (float)s;
    const float *src = row + (isk ? dim : 0) + 2 * pi;
    const float x0 = src[0], x1 = src[1];
    const float y0 = x0 * cf - x1 * sf, y1 = x0 * sf + x1 * cf;
    uint16_t *dst = (isk ? ko : qo) + 2 * pi;
    dst[0] = f32_to_bf16_bits(y0);
    dst[1] = f32_to_bf16_bits(y1);
  }
  const float *vsrc = row + dim + kvdim;
  for (int i = threadIdx.x; i < kvdim; i += blockDim.x) vo[i] = f32_to_bf16_bits(vsrc[i]);
}

// gu: f32 [B, 2*ffn] = (W1 x | W3 x); act = bf16(silu(g) * u)
__global__ void swiglu_kernel(const float *__restrict__ gu, int ffn, int total, uint16_t *__restrict__ act) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < total) {
    const int b = i / ffn, j = i % ffn;
    const float g = gu[(size_t)b * 2 * ffn + j], u = gu[(size_t)b * 2 * ffn + ffn + j];
    const float sg = g * (1.0f / (1.0f + expf(0.0f - g)));
    act[i] = f32_to_bf16_bits(sg * u);
  }
}

__global__ void embed_kernel(const uint16_t *__restrict__ emb, const int32_t *__restrict__ tokens, int dim, int vocab,
                             float *__restrict__ x) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const int b = blockIdx.x;
  int t = tokens[b];
  t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
  const uint16_t *e = emb + (size_t)t * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(size_t)b * dim + i] = bf16_bits_to_f32(e[i]);
}

__global__ void argmax_kernel(const float *__restrict__ logits, int vocab, int32_t *__restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const float *l = logits + (size_t)blockIdx.x * vocab;
  float best = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = l[i];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = sv[0];
    int ix = si[0];
    for (int w = 1; w < nw; w++)
      if (sv[w] > b || (sv[w] == b && si[w] < ix)) {
        b = sv[w];
        ix = si[w];
      }
    out[blockIdx.x] = ix == 0x7FFFFFFF ? 0 : ix;
  }
}

// Counter-based normal generator for synthetic weights: SplitMix64 of
// (seed, index) -> two uniforms -> Box-Muller.
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void normal_kernel(float *__restrict__ out, size_t n, uint64_t seed, size_t offset, float sigma) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t r = splitmix64(seed * 0x100000001B3ull + (offset + i));
  const float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
  const float u2 = (float)((r >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
  out[i] = sigma * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// The [rows, cols] block at (row0, col0) of the [*, ld] matrix that
// normal_kernel generates with the same seed (element index row * ld + col).
__global__ void normal_block_kernel(float *__restrict__ out, int rows, int cols, size_t row0, size_t col0, size_t ld,
                                    uint64_t seed, float sigma) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * cols) return;
  const size_t r = i / cols, c = i % cols;
  const uint64_t z = splitmix64(seed * 0x100000001B3ull + ((row0 + r) * ld + col0 + c));
  const float u1 = ((float)(z >> 40) + 0.5f) * (1.0f / 16777216.0f);
  const float u2 = (float)((z >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
  out[i] = sigma * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// Order-preserving key of (value, index) for a distributed first-max argmax:
// larger value wins, then the smaller index; 0 for NaN.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  if (v != v) return 0ull;
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (0xFFFFFFFFu - (uint32_t)idx);
}

// Key of the first maximum of each row of a vocab shard starting at `offset`.
__global__ void argmax_key_kernel(const float *__restrict__ logits, int vocab, int offset,
                                  unsigned long long *__restrict__ keys) {
  __shared__ unsigned long long sk[32];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const float *l = logits + (size_t)blockIdx.x * vocab;
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) best = max(best, argmax_key(l[i], offset + i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) sk[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = sk[0];
    for (int w = 1; w < nw; w++) b = max(b, sk[w]);
    keys[blockIdx.x] = b;
  }
}

__global__ void key_to_token_kernel(const unsigned long long *__restrict__ keys, int rows, int32_t *__restrict__ out) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows) out[i] = keys[i] == 0ull ? 0 : (int32_t)(0xFFFFFFFFu - (uint32_t)(keys[i] & 0xFFFFFFFFull));
}

// [tp][rows][shard] (all-gathered vocab shards) -> [rows][tp * shard]
__global__ void unshard_kernel(const float *__restrict__ in, int tp, int rows, int shard, float *__restrict__ out) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t n = (size_t)tp * rows * shard;
  if (i >= n) return;
  const int r = (int)(i / ((size_t)tp * shard));
  const size_t col = i % ((size_t)tp * shard);
  const int t = (int)(col / shard), c = (int)(col % shard);
  out[i] = in[((size_t)t * rows + r) * shard + c];
}

template <typename... Args>
int launch_pdl(vxb_ctx *ctx, void (*kfn)(Args...), dim3 grid, dim3 block, cudaStream_t st, const char *what,
               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, args...);
  if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  return VXB_OK;
}

}  // namespace

namespace vxb {

int rmsnorm_launch(vxb_ctx *ctx, const float *x, const float *w, const float *b, int rows, int n, float eps,
                   uint16_t *out, cudaStream_t st) {
  return launch_pdl(ctx, rmsnorm_kernel, dim3(rows), dim3(512), st, "rmsnorm_kernel", x, w, b, n, eps, out);
}

int rope_launch(vxb_ctx *ctx, const float *qkv, int rows, int dim, int kvdim, const KVPlace *places,
                const double *rope_div, uint16_t *q_out, uint16_t *k_out, uint16_t *v_out, cudaStream_t st,
                int q_pair0, int k_pair0) {
  return launch_pdl(ctx, rope_kernel, dim3(rows), dim3(512), st, "rope_kernel", qkv, dim, kvdim, places, rope_div,
                    q_out, k_out, v_out, q_pair0, k_pair0);
}

int swiglu_launch(vxb_ctx *ctx, const float *gu, int rows, int ffn, uint16_t *act, cudaStream_t st) {
  const int total = rows * ffn;
  return launch_pdl(ctx, swiglu_kernel, dim3((total + 255) / 256), dim3(256), st, "swiglu_kernel", gu, ffn, total,
                    act);
}

int embed_launch(vxb_ctx *ctx, const uint16_t *emb, const int32_t *tokens, int rows, int dim, int vocab, float *x,
                 cudaStream_t st) {
  return launch_pdl(ctx, embed_kernel, dim3(rows), dim3(512), st, "embed_kernel", emb, tokens, dim, vocab, x);
}

int argmax_launch(vxb_ctx *ctx, const float *logits, int rows, int vocab, int32_t *out, cudaStream_t st) {
  return launch_pdl(ctx, argmax_kernel, dim3(rows), dim3(1024), st, "argmax_kernel", logits, vocab, out);
}

int normal_fill(vxb_ctx *ctx, float *out, size_t n, uint64_t seed, size_t offset, float sigma, cudaStream_t st) {
  if (n == 0) return VXB_OK;
  normal_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(out, n, seed, offset, sigma);
  return launch_check(ctx, "normal_kernel");
}

int normal_fill_block(vxb_ctx *ctx, float *out, int rows, int cols, size_t row0, size_t col0, size_t ld, uint64_t seed,
                      float sigma, cudaStream_t st) {
  const size_t n = (size_t)rows * cols;
  if (n == 0) return VXB_OK;
  normal_block_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(out, rows, cols, row0, col0, ld, seed, sigma);
  return launch_check(ctx, "normal_block_kernel");
}

int argmax_key_launch(vxb_ctx *ctx, const float *logits, int rows, int vocab, int offset, unsigned long long *keys,
                      cudaStream_t st) {
  return launch_pdl(ctx, argmax_key_kernel, dim3(rows), dim3(1024), st, "argmax_key_kernel", logits, vocab, offset,
                    keys);
}

int key_to_token_launch(vxb_ctx *ctx, const unsigned long long *keys, int rows, int32_t *out, cudaStream_t st) {
  return launch_pdl(ctx, key_to_token_kernel, dim3((rows + 127) / 128), dim3(128), st, "key_to_token_kernel", keys,
                    rows, out);
}

int unshard_launch(vxb_ctx *ctx, const float *in, int tp, int rows, int shard, float *out, cudaStream_t st) {
  const size_t n = (size_t)tp * rows * shard;
  unshard_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(in, tp, rows, shard, out);
  return launch_check(ctx, "unshard_kernel");
}

}  // namespace vxb

// ---- standalone entry points (used by tests and by callers of single ops)

VXB_API int vxb_rmsnorm(vxb_ctx *ctx, const float *d_x, const float *d_w, const float *d_b, int rows, int n, float eps,
                        uint16_t *d_out, void *stream) {
  if (!ctx || !d_x || !d_w || !d_b || !d_out || rows <= 0 || n <= 0)
    return set_error(ctx, VXB_EINVAL, "vxb_rmsnorm: bad arguments");
  if (int rc = use_device(ctx)) return rc;
  return rmsnorm_launch(ctx, d_x, d_w, d_b, rows, n, eps, d_out, (cudaStream_t)stream);
}

VXB_API int vxb_swiglu(vxb_ctx *ctx, const float *d_gu, int rows, int ffn, uint16_t *d_act, void *stream) {
  if (!ctx || !d_gu || !d_act || rows <= 0 || ffn <= 0) return set_error(ctx, VXB_EINVAL, "vxb_swiglu: bad arguments");
  if (int rc = use_device(ctx)) return rc;
  return swiglu_launch(ctx, d_gu, rows, ffn, d_act, (cudaStream_t)stream);
}

VXB_API int vxb_argmax(vxb_ctx *ctx, const float *d_logits, int rows, int vocab, int32_t *d_out, void *stream) {
  if (!ctx || !d_logits || !d_out || rows <= 0 || vocab <= 0) return set_error(ctx, VXB_EINVAL, "vxb_argmax: bad arguments");
  if (int rc = use_device(ctx)) return rc;
  return argmax_launch(ctx, d_logits, rows, vocab, d_out, (cudaStream_t)stream);
}
