// K5: the small per-token kernels of the Llama-style decoder block
// (stdlib/ai/transformer.vx:413-603):
//   rmsnorm_bias : x * w / sqrt(mean(x^2) + eps) + b            (413-439)
//   rope         : adjacent pairs (x[2i], x[2i+1]) of the whole projection
//                  rotated by theta = pos / exp(i * ln(10000) / dim) (442-466)
//   swiglu       : silu(W1 x) * (W3 x), silu(x) = x * sigmoid(x)   (591-603, 176-182)
//   embed        : token embedding row -> f32 residual stream
//   argmax       : greedy next token, first index of the maximum (1163-1177)
// Accumulation is f32; the GEMV inputs are rounded once to bf16.
// Every kernel is launched with programmatic stream serialization and lets
// the next kernel of the stream launch as soon as it starts, so a chain of
// small kernels and GEMVs launches ahead and each GEMV prefetches its weights
// while earlier kernels run. Each kernel waits for its predecessor to
// complete before reading anything produced on the device, and reads such
// data through L2 only (ld.global.cg): with kernels launched ahead, an SM's
// L1 can still hold lines that an earlier, concurrently running kernel read
// before a later kernel rewrote them.
#include <cuda_bf16.h>

#include <algorithm>

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

// One CTA (512 threads) per row. Rows whose length is a multiple of 4 and at
// most 8192 are read once with 16-byte loads into registers (w and b are
// requested before the wait on the producing kernel), so the kernel costs one
// memory round trip and one block reduction.
constexpr int NORM_THREADS = 512;
constexpr int NORM_VEC = 4;  // float4 per thread

__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                               const float *__restrict__ b, int n, float eps,
                                                               uint16_t *__restrict__ out) {
  __shared__ float red[32];
  const float *xr = x + (size_t)blockIdx.x * n;
  uint16_t *o = out + (size_t)blockIdx.x * n;
  const int nv = n >> 2;
  if ((n & 3) == 0 && nv <= NORM_VEC * NORM_THREADS) {
    const float4 *x4 = reinterpret_cast<const float4 *>(xr);
    const float4 *w4 = reinterpret_cast<const float4 *>(w), *b4 = reinterpret_cast<const float4 *>(b);
    float4 xv[NORM_VEC], wv[NORM_VEC], bv[NORM_VEC];
#pragma unroll
    for (int u = 0; u < NORM_VEC; u++) {
      const int i = threadIdx.x + u * NORM_THREADS;
      if (i < nv) {
        wv[u] = __ldg(w4 + i);
        bv[u] = __ldg(b4 + i);
      }
    }
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < NORM_VEC; u++) {
      const int i = threadIdx.x + u * NORM_THREADS;
      if (i < nv) xv[u] = __ldcg(x4 + i);
    }
#pragma unroll
    for (int u = 0; u < NORM_VEC; u++) {
      const int i = threadIdx.x + u * NORM_THREADS;
      if (i < nv) {
        ss = fmaf(xv[u].x, xv[u].x, ss);
        ss = fmaf(xv[u].y, xv[u].y, ss);
        ss = fmaf(xv[u].z, xv[u].z, ss);
        ss = fmaf(xv[u].w, xv[u].w, ss);
      }
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
#pragma unroll
    for (int u = 0; u < NORM_VEC; u++) {
      const int i = threadIdx.x + u * NORM_THREADS;
      if (i < nv) {
        uint2 r;
        r.x = (uint32_t)f32_to_bf16_bits(xv[u].x * inv * wv[u].x + bv[u].x) |
              ((uint32_t)f32_to_bf16_bits(xv[u].y * inv * wv[u].y + bv[u].y) << 16);
        r.y = (uint32_t)f32_to_bf16_bits(xv[u].z * inv * wv[u].z + bv[u].z) |
              ((uint32_t)f32_to_bf16_bits(xv[u].w * inv * wv[u].w + bv[u].w) << 16);
        *reinterpret_cast<uint2 *>(o + 4 * i) = r;
      }
    }
    return;
  }
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = __ldcg(xr + i);
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = f32_to_bf16_bits(__ldcg(xr + i) * inv * w[i] + b[i]);
}

// RoPE of the new token(s) fused with the KV-cache append. One CTA per
// (row, head slot), hd/2 threads (one rotation pair each): slots [0, hq)
// rotate query heads into q_out (bf16 [rows, hq*hd]); [hq, hq + hkv) rotate
// key heads and [hq + hkv, hq + 2*hkv) round value heads to bf16, both
// written into the paged cache at the row's place (bf16, or int8 with the
// per-(token, head) absmax scale of append_token) and, when k_lin / v_lin
// are given, into [rows, hkv*hd] buffers. The rotation angle is
// pos / rope_div[pair] in f64 (pairs numbered from q_pair0 / k_pair0 for a
// tensor-parallel slice of the heads); the rotation itself is f32.
struct RopeKVArgs {
  const float *qkv;  // f32 [rows, qdim + 2*kvdim] = (q | k | v)
  const KVPlace *places;
  const double *rope_div;
  uint16_t *q_out, *k_lin, *v_lin;
  int qdim, kvdim, hd, hq, hkv, q_pair0, k_pair0;
  // cache (pool_k null: no cache write)
  int layer, bs, max_seqs, mbps, is_int8;
  void *pool_k, *pool_v;
  float *scale_k, *scale_v;
  int32_t *tables, *lens;
};

__global__ void rope_kv_kernel(const RopeKVArgs a) {
  __shared__ double red[32];
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int r = blockIdx.x, slot = blockIdx.y, t = threadIdx.x;
  const int4 pv = __ldcg(reinterpret_cast<const int4 *>(a.places + r));
  const KVPlace p = {pv.x, pv.y, pv.z, pv.w};
  const int kind = slot < a.hq ? 0 : (slot < a.hq + a.hkv ? 1 : 2);  // q, k, v
  const int h = kind == 0 ? slot : (kind == 1 ? slot - a.hq : slot - a.hq - a.hkv);
  const float *row = a.qkv + (size_t)r * (a.qdim + 2 * a.kvdim);
  const float2 xin =
      __ldcg(reinterpret_cast<const float2 *>(row + (kind == 0 ? 0 : (kind == 1 ? a.qdim : a.qdim + a.kvdim)) + h * a.hd + 2 * t));
  float y0 = xin.x, y1 = xin.y;
  if (kind < 2) {
    const int pi = h * (a.hd / 2) + t;
    double s, c;
    sincos((double)p.pos / a.rope_div[pi + (kind ? a.k_pair0 : a.q_pair0)], &s, &c);
    const float cf = (float)c, sf = (float)s;
    const float x0 = xin.x, x1 = xin.y;
    y0 = x0 * cf - x1 * sf;
    y1 = x0 * sf + x1 * cf;
  }
  const uint32_t packed = (uint32_t)f32_to_bf16_bits(y0) | ((uint32_t)f32_to_bf16_bits(y1) << 16);
  if (kind == 0) {
    *reinterpret_cast<uint32_t *>(a.q_out + (size_t)r * a.qdim + h * a.hd + 2 * t) = packed;
    return;
  }
  uint16_t *lin = kind == 1 ? a.k_lin : a.v_lin;
  if (lin) *reinterpret_cast<uint32_t *>(lin + (size_t)r * a.kvdim + h * a.hd + 2 * t) = packed;
  if (!a.pool_k) return;
  const size_t tok = ((size_t)p.block * a.hkv + h) * a.bs + p.offset;
  if (!a.is_int8) {
    uint16_t *pool = reinterpret_cast<uint16_t *>(kind == 1 ? a.pool_k : a.pool_v);
    *reinterpret_cast<uint32_t *>(pool + tok * a.hd + 2 * t) = packed;
  } else {
    // absmax of the head's bf16 values in f64, scale absmax/127 (1 when all
    // zero), codes round-half-away(v / scale) clamped to [-128, 127]
    const double v0 = (double)bf16_bits_to_f32(packed & 0xFFFFu), v1 = (double)bf16_bits_to_f32(packed >> 16);
    double m = fmax(fabs(v0), fabs(v1));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int warp = t >> 5, nw = (blockDim.x + 31) >> 5;
    if ((t & 31) == 0) red[warp] = m;
    __syncthreads();
    for (int i = 0; i < nw; i++) m = fmax(m, red[i]);
    const double scale = m == 0.0 ? 1.0 : m / 127.0;
    const double q0 = round(v0 / scale), q1 = round(v1 / scale);
    const int8_t c0 = (int8_t)(isnan(q0) ? 0.0 : fmin(fmax(q0, -128.0), 127.0));
    const int8_t c1 = (int8_t)(isnan(q1) ? 0.0 : fmin(fmax(q1, -128.0), 127.0));
    int8_t *pool = reinterpret_cast<int8_t *>(kind == 1 ? a.pool_k : a.pool_v);
    *reinterpret_cast<uint16_t *>(pool + tok * a.hd + 2 * t) = (uint16_t)((uint8_t)c0 | ((uint16_t)(uint8_t)c1 << 8));
    if (t == 0) (kind == 1 ? a.scale_k : a.scale_v)[tok] = (float)scale;
  }
  if (kind == 1 && h == 0 && t == 0) {
    if (p.offset == 0) a.tables[((size_t)a.layer * a.max_seqs + p.slot) * a.mbps + p.pos / a.bs] = p.block;
    atomicMax(a.lens + (size_t)a.layer * a.max_seqs + p.slot, p.pos + 1);
  }
}

// gu: f32 [B, 2*ffn] = (W1 x | W3 x); act = bf16(silu(g) * u)
__global__ void swiglu_kernel(const float *__restrict__ gu, int ffn, int total, uint16_t *__restrict__ act) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < total) {
    const int b = i / ffn, j = i % ffn;
    const float g = __ldcg(gu + (size_t)b * 2 * ffn + j), u = __ldcg(gu + (size_t)b * 2 * ffn + ffn + j);
    const float sg = g * (1.0f / (1.0f + expf(0.0f - g)));
    act[i] = f32_to_bf16_bits(sg * u);
  }
}

__global__ void embed_kernel(const uint16_t *__restrict__ emb, const int32_t *__restrict__ tokens, int dim, int vocab,
                             float *__restrict__ x) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.x;
  int t = __ldcg(tokens + b);
  t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
  const uint16_t *e = emb + (size_t)t * dim;
  float *xr = x + (size_t)b * dim;
  if ((dim & 7) == 0) {
    for (int i = threadIdx.x; i < dim / 8; i += blockDim.x) {
      const uint4 v = __ldg(reinterpret_cast<const uint4 *>(e) + i);
      float4 *o = reinterpret_cast<float4 *>(xr) + 2 * i;
      o[0] = make_float4(bf16_bits_to_f32(v.x & 0xFFFFu), bf16_bits_to_f32(v.x >> 16), bf16_bits_to_f32(v.y & 0xFFFFu),
                         bf16_bits_to_f32(v.y >> 16));
      o[1] = make_float4(bf16_bits_to_f32(v.z & 0xFFFFu), bf16_bits_to_f32(v.z >> 16), bf16_bits_to_f32(v.w & 0xFFFFu),
                         bf16_bits_to_f32(v.w >> 16));
    }
    return;
  }
  for (int i = threadIdx.x; i < dim; i += blockDim.x) xr[i] = bf16_bits_to_f32(e[i]);
}

// Rows whose length is a multiple of 4 are scanned with 16-byte loads, eight
// per thread in flight; indices seen by one thread ascend, so the first
// maximum wins by the (value, index) comparison below.
template <typename Visit>
__device__ __forceinline__ void scan_row(const float *__restrict__ l, int vocab, Visit visit) {
  if ((vocab & 3) == 0) {
    const float4 *l4 = reinterpret_cast<const float4 *>(l);
    const int nv = vocab >> 2;
    for (int base = threadIdx.x; base < nv; base += 8 * blockDim.x) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int i = base + u * blockDim.x;
        if (i < nv) v[u] = __ldcg(l4 + i);
      }
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int i = base + u * blockDim.x;
        if (i < nv) {
          visit(v[u].x, 4 * i);
          visit(v[u].y, 4 * i + 1);
          visit(v[u].z, 4 * i + 2);
          visit(v[u].w, 4 * i + 3);
        }
      }
    }
    return;
  }
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) visit(__ldcg(l + i), i);
}

__global__ void __launch_bounds__(1024) argmax_kernel(const float *__restrict__ logits, int vocab, int32_t *__restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float *l = logits + (size_t)blockIdx.x * vocab;
  float best = -INFINITY;
  int bi = 0x7FFFFFFF;
  scan_row(l, vocab, [&](float v, int i) {
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  });
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
__global__ void __launch_bounds__(1024) argmax_key_kernel(const float *__restrict__ logits, int vocab, int offset,
                                                          unsigned long long *__restrict__ keys) {
  __shared__ unsigned long long sk[32];
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const float *l = logits + (size_t)blockIdx.x * vocab;
  unsigned long long best = 0ull;
  scan_row(l, vocab, [&](float v, int i) { best = max(best, argmax_key(v, offset + i)); });
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
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows) {
    const unsigned long long k = __ldcg(keys + i);
    out[i] = k == 0ull ? 0 : (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
  }
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

// Standalone RoPE of f32 rows: one thread per adjacent pair (x[2i], x[2i+1])
// of a row, an odd last element copied. The angle is
// pos[row] / exp(i * ln(10000) / dim) (rope_embed,
// stdlib/ai/transformer.vx:442-466) when by_angle is 0, else angles[i], and
// 0 for i >= n_angles (the `rope` builtin, src/interpreter.rs:2368-2373). The
// rotation is evaluated in f64 and rounded to f32 once. out may equal x: each
// element is read and written by the same thread.
__global__ void rope_rows_kernel(const float *x, const int64_t *__restrict__ pos, int dim, int by_angle,
                                 const double *__restrict__ angles, int n_angles, int rows, int n, float *out) {
  const size_t half = (size_t)(n + 1) / 2, total = (size_t)rows * half;
  const double ln_base = log(10000.0);
  for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
    const size_t r = g / half, i = g % half;
    const float *xr = x + r * n;
    float *orow = out + r * n;
    if (2 * i + 1 == (size_t)n) {
      orow[2 * i] = xr[2 * i];
      continue;
    }
    const double theta = by_angle ? (i < (size_t)n_angles ? angles[i] : 0.0)
                                : (double)pos[r] / exp((double)i * ln_base / (double)dim);
    double s, c;
    sincos(theta, &s, &c);
    const double x0 = xr[2 * i], x1 = xr[2 * i + 1];
    orow[2 * i] = (float)(x0 * c - x1 * s);
    orow[2 * i + 1] = (float)(x0 * s + x1 * c);
  }
}

// Residual add (_vec_add, stdlib/ai/transformer.vx:353-366): out = a + b in
// f32, 16-byte accesses when all three pointers allow them. out may equal a
// or b.
__global__ void add_kernel(const float *a, const float *b, size_t n, float *out) {
  const bool vec = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                     reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  const size_t n4 = vec ? n / 4 : 0, stride = (size_t)gridDim.x * blockDim.x;
  const size_t t0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (size_t i = t0; i < n4; i += stride) {
    const float4 va = __ldcs(reinterpret_cast<const float4 *>(a) + i);
    const float4 vb = __ldcs(reinterpret_cast<const float4 *>(b) + i);
    __stcs(reinterpret_cast<float4 *>(out) + i, make_float4(va.x + vb.x, va.y + vb.y, va.z + vb.z, va.w + vb.w));
  }
  for (size_t i = 4 * n4 + t0; i < n; i += stride) out[i] = a[i] + b[i];
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
  return launch_pdl(ctx, rmsnorm_kernel, dim3(rows), dim3(NORM_THREADS), st, "rmsnorm_kernel", x, w, b, n, eps, out);
}

int rope_kv_launch(vxb_ctx *ctx, vxb_kv *kv, int layer, const float *qkv, int rows, int qdim, int kvdim, int hd,
                   const KVPlace *places, const double *rope_div, uint16_t *q_out, uint16_t *k_lin, uint16_t *v_lin,
                   int q_pair0, int k_pair0, cudaStream_t st) {
  if (rows <= 0) return VXB_OK;
  if (hd % 64 || qdim % hd || kvdim % hd)
    return set_error(ctx, VXB_EINVAL, "rope_kv: head_dim %d must be a multiple of 64 dividing %d and %d", hd, qdim, kvdim);
  RopeKVArgs a = {};
  a.qkv = qkv;
  a.places = places;
  a.rope_div = rope_div;
  a.q_out = q_out;
  a.k_lin = k_lin;
  a.v_lin = v_lin;
  a.qdim = qdim;
  a.kvdim = kvdim;
  a.hd = hd;
  a.hq = qdim / hd;
  a.hkv = kvdim / hd;
  a.q_pair0 = q_pair0;
  a.k_pair0 = k_pair0;
  a.layer = layer;
  if (kv) {
    if (kv->num_kv_heads != a.hkv || kv->head_dim != hd)
      return set_error(ctx, VXB_EINVAL, "rope_kv: cache holds %d heads of %d, projections %d of %d", kv->num_kv_heads,
                       kv->head_dim, a.hkv, hd);
    a.bs = kv->block_size;
    a.max_seqs = kv->max_seqs;
    a.mbps = kv->max_blocks_per_seq;
    a.is_int8 = kv->dtype == VXB_I8;
    a.pool_k = kv->pool_k;
    a.pool_v = kv->pool_v;
    a.scale_k = kv->scale_k;
    a.scale_v = kv->scale_v;
    a.tables = kv->d_tables;
    a.lens = kv->d_lens;
  }
  return launch_pdl(ctx, rope_kv_kernel, dim3(rows, a.hq + 2 * a.hkv), dim3(hd / 2), st, "rope_kv_kernel", a);
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

static int rope_rows(vxb_ctx *ctx, const float *d_x, int rows, int n, const int64_t *d_pos, int dim, int by_angle,
                     const double *d_angles, int n_angles, float *d_out, cudaStream_t st) {
  if (int rc = use_device(ctx)) return rc;
  const size_t total = (size_t)rows * ((size_t)(n + 1) / 2);
  const size_t cap = (size_t)(ctx->num_sms > 0 ? ctx->num_sms : 148) * 8;
  const unsigned grid = (unsigned)std::max<size_t>(1, std::min((total + 255) / 256, cap));
  rope_rows_kernel<<<grid, 256, 0, st>>>(d_x, d_pos, dim, by_angle, d_angles, n_angles, rows, n, d_out);
  return launch_check(ctx, "rope_rows_kernel");
}

VXB_API int vxb_rope(vxb_ctx *ctx, const float *d_x, int rows, int n, const int64_t *d_pos, int dim, float *d_out,
                     void *stream) {
  if (!ctx || rows < 0 || n < 0 || dim <= 0) return set_error(ctx, VXB_EINVAL, "vxb_rope: bad arguments");
  if (rows == 0 || n == 0) return VXB_OK;  // an empty input rotates to an empty output
  if (!d_x || !d_pos || !d_out) return set_error(ctx, VXB_EINVAL, "vxb_rope: null pointer");
  return rope_rows(ctx, d_x, rows, n, d_pos, dim, 0, nullptr, 0, d_out, (cudaStream_t)stream);
}

VXB_API int vxb_rope_angles(vxb_ctx *ctx, const float *d_x, int rows, int n, const double *d_angles, int n_angles,
                            float *d_out, void *stream) {
  if (!ctx || rows < 0 || n < 0 || n_angles < 0 || (n_angles > 0 && !d_angles))
    return set_error(ctx, VXB_EINVAL, "vxb_rope_angles: bad arguments");
  if (rows == 0 || n == 0) return VXB_OK;
  if (!d_x || !d_out) return set_error(ctx, VXB_EINVAL, "vxb_rope_angles: null pointer");
  return rope_rows(ctx, d_x, rows, n, nullptr, 1, 1, d_angles, n_angles, d_out, (cudaStream_t)stream);
}

VXB_API int vxb_add(vxb_ctx *ctx, const float *d_a, const float *d_b, size_t n, float *d_out, void *stream) {
  if (!ctx) return set_error(ctx, VXB_EINVAL, "vxb_add: bad arguments");
  if (n == 0) return VXB_OK;  // _vec_add of two empty vectors is empty
  if (!d_a || !d_b || !d_out) return set_error(ctx, VXB_EINVAL, "vxb_add: null pointer");
  if (int rc = use_device(ctx)) return rc;
  const size_t cap = (size_t)(ctx->num_sms > 0 ? ctx->num_sms : 148) * 8;
  const unsigned grid = (unsigned)std::max<size_t>(1, std::min((n / 4 + 255) / 256, cap));
  add_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(d_a, d_b, n, d_out);
  return launch_check(ctx, "add_kernel");
}

VXB_API int vxb_argmax(vxb_ctx *ctx, const float *d_logits, int rows, int vocab, int32_t *d_out, void *stream) {
  if (!ctx || !d_logits || !d_out || rows <= 0 || vocab <= 0) return set_error(ctx, VXB_EINVAL, "vxb_argmax: bad arguments");
  if (int rc = use_device(ctx)) return rc;
  return argmax_launch(ctx, d_logits, rows, vocab, d_out, (cudaStream_t)stream);
}
