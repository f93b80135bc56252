// Weight blocks: host codec, device quantizer/dequantizer, and the tiled HBM
// layout used by the GEMV/GEMM kernels.
//
// Block format (gguf_loader.rs, src/gguf_loader.rs:413-498):
//   Q8_0: 34 bytes = f16 d (little endian) + 32 x int8 code, x = code * d
//   Q4_0: 18 bytes = f16 d + 16 bytes; byte j holds element 2j in its low
//         nibble and 2j+1 in its high nibble, x = (nibble - 8) * d
// Codes: QuantTensor::quantize PerGroup, group 32 over the flat buffer
// (src/quantize.rs:96-163): scale = absmax/127 (INT8) or absmax/8 (INT4,
// calibrate_minmax_range, 594-600), all-zero group -> 1.0; code =
// clamp(round_half_away(v/scale), qmin, qmax). The f64 scale is stored as
// f32_to_f16((float)scale) (tensor_engine.rs:42-64, truncating).
#include <cmath>
#include <cstring>
#include <vector>

#include "tiled_layout.h"
#include "vxb_internal.h"

using namespace vxb;

namespace {

// ---------------- host codec ----------------

uint16_t host_f32_to_f16_trunc(float x) {
  uint32_t bits;
  std::memcpy(&bits, &x, 4);
  uint32_t sign = (bits >> 16) & 0x8000u;
  int exp = (int)((bits >> 23) & 0xFFu);
  uint32_t frac = bits & 0x7FFFFFu;
  if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (frac != 0 ? 0x200u : 0u));
  int ne = exp - 127 + 15;
  if (ne >= 31) return (uint16_t)(sign | 0x7C00u);
  if (ne <= 0) {
    if (ne < -10) return (uint16_t)sign;
    uint32_t f = (frac | 0x800000u) >> (uint32_t)(1 - ne);
    return (uint16_t)(sign | (f >> 13));
  }
  return (uint16_t)(sign | ((uint32_t)ne << 10) | (frac >> 13));
}

float host_ref_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t frac = h & 0x3FFu;
  uint32_t out;
  if (exp == 0) {
    if (frac == 0) {
      out = sign;
    } else {
      int e = 0;
      uint32_t f = frac;
      while ((f & 0x400u) == 0) {
        f <<= 1;
        e++;
      }
      out = sign | ((uint32_t)(127 - 15 - e) << 23) | ((f & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    out = sign | 0x7F800000u | (frac << 13);
  } else {
    out = sign | ((exp + 112u) << 23) | (frac << 13);
  }
  float r;
  std::memcpy(&r, &out, 4);
  return r;
}

int code_of(double v, double scale, int qmin, int qmax) {
  if (scale == 0.0) return 0;
  double r = std::round(v / scale);
  if (std::isnan(r)) return 0;
  if (r < qmin) return qmin;
  if (r > qmax) return qmax;
  return (int)r;
}

template <typename T>
int pack_blocks_host(int fmt, const T *w, size_t n, uint8_t *out) {
  const bool q4 = fmt == VXB_Q4_0;
  const size_t nb = (n + 31) / 32, bb = q4 ? 18 : 34;
  for (size_t b = 0; b < nb; b++) {
    size_t s = b * 32, len = s + 32 <= n ? 32 : n - s;
    double amax = 0.0;
    for (size_t i = 0; i < len; i++) amax = std::fmax(amax, std::fabs((double)w[s + i]));
    double scale = amax == 0.0 ? 1.0 : amax / (q4 ? 8.0 : 127.0);
    uint16_t h = host_f32_to_f16_trunc((float)scale);
    uint8_t *blk = out + b * bb;
    blk[0] = (uint8_t)(h & 0xFF);
    blk[1] = (uint8_t)(h >> 8);
    int q[32];
    for (size_t i = 0; i < 32; i++) q[i] = i < len ? code_of((double)w[s + i], scale, q4 ? -8 : -128, q4 ? 7 : 127) : 0;
    if (q4) {
      for (int j = 0; j < 16; j++)
        blk[2 + j] = (uint8_t)(((q[2 * j] & 0xF) ^ 0x8) | (((q[2 * j + 1] & 0xF) ^ 0x8) << 4));
    } else {
      for (int j = 0; j < 32; j++) blk[2 + j] = (uint8_t)(int8_t)q[j];
    }
  }
  return VXB_OK;
}

// ---------------- device quantizer / dequantizer ----------------

// One warp per 32-element block.
__global__ void quantize_blocks_kernel(const float *__restrict__ w, size_t n, uint8_t *__restrict__ out,
                                       int q4) {
  const size_t blk = (size_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const size_t nb = (n + 31) / 32;
  if (blk >= nb) return;
  const size_t idx = blk * 32 + lane;
  const bool valid = idx < n;
  const double v = valid ? (double)w[idx] : 0.0;
  double a = valid ? fabs(v) : 0.0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmax(a, __shfl_xor_sync(0xffffffffu, a, o));
  const double scale = a == 0.0 ? 1.0 : a / (q4 ? 8.0 : 127.0);
  int q = 0;
  if (valid && scale != 0.0) {
    double r = round(v / scale);
    const double qmin = q4 ? -8.0 : -128.0, qmax = q4 ? 7.0 : 127.0;
    q = isnan(r) ? 0 : (int)fmin(fmax(r, qmin), qmax);
  }
  const uint16_t h = f32_to_f16_trunc(__double2float_rn(scale));
  if (q4) {
    uint8_t *b = out + blk * 18;
    const int nib = (q & 0xF) ^ 0x8;
    const int hi = __shfl_down_sync(0xffffffffu, nib, 1);
    if ((lane & 1) == 0) b[2 + lane / 2] = (uint8_t)(nib | (hi << 4));
    if (lane == 0) {
      b[0] = (uint8_t)(h & 0xFF);
      b[1] = (uint8_t)(h >> 8);
    }
  } else {
    uint8_t *b = out + blk * 34;
    b[2 + lane] = (uint8_t)(int8_t)q;
    if (lane == 0) {
      b[0] = (uint8_t)(h & 0xFF);
      b[1] = (uint8_t)(h >> 8);
    }
  }
}

__global__ void dequantize_blocks_kernel(const uint8_t *__restrict__ blocks, size_t n, float *__restrict__ out,
                                         int q4) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const size_t b = i / 32, e = i % 32;
  if (q4) {
    const uint8_t *blk = blocks + b * 18;
    const float d = ref_f16_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
    const uint8_t byte = blk[2 + e / 2];
    const int nib = (e & 1) ? (byte >> 4) : (byte & 0xF);
    out[i] = (float)(nib - 8) * d;
  } else {
    const uint8_t *blk = blocks + b * 34;
    const float d = ref_f16_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
    out[i] = (float)(int8_t)blk[2 + e] * d;
  }
}

// GGUF types beyond the kernels' storage formats (src/gguf_loader.rs:443-531):
// Q4_1 (20 bytes: f16 d, f16 m, 16 nibble bytes; x = nibble * d + m with the
// multiply and the add rounded separately), F16 (the reference's f16_to_f32,
// subnormals included) and F32 (the bytes as they are).
__global__ void dequantize_ggml_kernel(const uint8_t *__restrict__ data, size_t n, float *__restrict__ out, int type) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (type == VXB_Q4_1) {
    const uint8_t *blk = data + (i / 32) * 20;
    const float d = ref_f16_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
    const float m = ref_f16_to_f32((uint32_t)blk[2] | ((uint32_t)blk[3] << 8));
    const uint8_t byte = blk[4 + (i % 32) / 2];
    const int nib = (i & 1) ? (byte >> 4) : (byte & 0xF);
    out[i] = __fadd_rn(__fmul_rn((float)nib, d), m);
  } else if (type == VXB_GGML_F16) {
    out[i] = ref_f16_to_f32((uint32_t)data[2 * i] | ((uint32_t)data[2 * i + 1] << 8));
  } else {
    out[i] = __uint_as_float((uint32_t)data[4 * i] | ((uint32_t)data[4 * i + 1] << 8) |
                             ((uint32_t)data[4 * i + 2] << 16) | ((uint32_t)data[4 * i + 3] << 24));
  }
}

// ---------------- tiled layout ----------------

__global__ void tile_header_kernel(uint32_t *hdr, int fmt, int N, int K) {
  hdr[0] = TILED_MAGIC;
  hdr[2] = (uint32_t)fmt;
  hdr[3] = (uint32_t)N;
  hdr[4] = (uint32_t)K;
}

__device__ __forceinline__ uint32_t q4_nibble(const uint8_t *blocks, int N, int K, int r, int k) {
  if (r >= N || k >= K) return 8u;
  const uint8_t *blk = blocks + ((size_t)r * (K / 32) + k / 32) * 18;
  const uint8_t byte = blk[2 + (k % 32) / 2];
  return (k & 1) ? (byte >> 4) : (byte & 0xF);
}

__device__ __forceinline__ uint32_t q8_byte(const uint8_t *blocks, int N, int K, int r, int k) {
  if (r >= N || k >= K) return 0u;
  return blocks[((size_t)r * (K / 32) + k / 32) * 34 + 2 + (k % 32)];
}

// One thread per u32 of the codes of the part's tiles. `blocks` holds the N
// source rows of the part, which land at tiles [tile0, tile0 + ceil(N/16)) of
// a layout of geometry g (the whole, possibly fused, matrix).
__global__ void tile_codes_kernel(const uint8_t *__restrict__ blocks, int fmt, int N, int K, TiledGeom g, int tile0,
                                  uint8_t *__restrict__ tiled) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t total = (size_t)((N + 15) / 16) * g.n_chunks * 128;
  if (idx >= total) return;
  const int j = idx % 4;
  const int l = (idx / 4) % 32;
  const size_t tc = idx / 128;  // (tile, chunk) of the part
  const int c = (int)(tc % g.n_chunks);
  const int t = (int)(tc / g.n_chunks);
  // k-permuted fragments: lane q of a k16 step holds columns 4q..4q+3, so the
  // activation operand of the lane is 8 contiguous bytes
  const int r0 = t * 16 + l / 4, r1 = r0 + 8, k4 = (l % 4) * 4;
  uint32_t w = 0;
  if (fmt == VXB_Q4_0) {
    const int kb = (4 * c + j) * 16 + k4;
    w = q4_nibble(blocks, N, K, r0, kb) | (q4_nibble(blocks, N, K, r1, kb) << 4) |
        (q4_nibble(blocks, N, K, r0, kb + 2) << 8) | (q4_nibble(blocks, N, K, r1, kb + 2) << 12) |
        (q4_nibble(blocks, N, K, r0, kb + 1) << 16) | (q4_nibble(blocks, N, K, r1, kb + 1) << 20) |
        (q4_nibble(blocks, N, K, r0, kb + 3) << 24) | (q4_nibble(blocks, N, K, r1, kb + 3) << 28);
  } else {
    // int8 codes are stored offset by 128 (q ^ 0x80)
    const int kb = (2 * c + j / 2) * 16 + k4 + ((j & 1) ? 2 : 0);
    w = q8_byte(blocks, N, K, r0, kb) | (q8_byte(blocks, N, K, r0, kb + 1) << 8) |
        (q8_byte(blocks, N, K, r1, kb) << 16) | (q8_byte(blocks, N, K, r1, kb + 1) << 24);
    w ^= 0x80808080u;
  }
  *reinterpret_cast<uint32_t *>(tiled + tiled_codes_at(g, tile0 + t, c) + l * 16 + j * 4) = w;
}

// One thread per u32 of the part's scales, ordered (tile, chunk, i, block of
// the chunk): entry = f16 scale of row 16t+i (low half) | row 16t+i+8 (high).
__global__ void tile_scales_kernel(const uint8_t *__restrict__ blocks, int fmt, int N, int K, TiledGeom g, int tile0,
                                   uint8_t *__restrict__ tiled) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t total = (size_t)((N + 15) / 16) * g.n_blocks * 8;
  if (idx >= total) return;
  const int bpc = g.chunk / 32;
  const int bb = idx % bpc;
  const int i = (idx / bpc) % 8;
  const size_t tc = idx / (8 * bpc);
  const int c = (int)(tc % g.n_chunks);
  const int t = (int)(tc / g.n_chunks);
  const int b = c * bpc + bb;
  const size_t blk_bytes = fmt == VXB_Q4_0 ? 18 : 34;
  uint32_t out = 0;
  bool sub = false;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int r = t * 16 + i + 8 * h;
    uint32_t s = 0;
    if (r < N && b < K / 32) {
      const uint8_t *blk = blocks + ((size_t)r * (K / 32) + b) * blk_bytes;
      s = (uint32_t)blk[0] | ((uint32_t)blk[1] << 8);
      if ((s & 0x7C00u) == 0 && (s & 0x3FFu) != 0) sub = true;
    }
    out |= s << (16 * h);
  }
  *reinterpret_cast<uint32_t *>(tiled + tiled_scales_at(g, tile0 + t, c) + (i * bpc + bb) * 4) = out;
  if (sub) atomicOr(reinterpret_cast<uint32_t *>(tiled) + 1, TILED_FLAG_SUBNORMAL_SCALES);
}

// One thread per (row, block): rebuild the GGUF block from the tiled layout.
__global__ void untile_kernel(const uint8_t *__restrict__ tiled, int fmt, int N, int K, TiledGeom g,
                              uint8_t *__restrict__ blocks) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int nbk = K / 32;
  if (idx >= (size_t)N * nbk) return;
  const int r = (int)(idx / nbk), b = (int)(idx % nbk);
  const int t = r / 16, ri = r % 16;
  const int bpc = g.chunk / 32;
  const uint32_t s =
      *reinterpret_cast<const uint32_t *>(tiled + tiled_scales_at(g, t, b / bpc) + ((ri & 7) * bpc + b % bpc) * 4) >>
      (ri >= 8 ? 16 : 0);
  if (fmt == VXB_Q4_0) {
    uint8_t *o = blocks + idx * 18;
    o[0] = (uint8_t)(s & 0xFF);
    o[1] = (uint8_t)((s >> 8) & 0xFF);
    for (int jb = 0; jb < 16; jb++) {
      uint32_t nib[2];
      for (int e = 0; e < 2; e++) {
        const int k = b * 32 + 2 * jb + e;
        const int step = k / 16, kk = k % 16;
        const int c = step / 4, j = step % 4;
        const int jj = kk & 3, lane = (ri & 7) * 4 + kk / 4;
        const int pos = (ri >= 8 ? 4 : 0) + (jj >= 2 ? 8 : 0) + ((jj & 1) ? 16 : 0);
        const uint32_t w = *reinterpret_cast<const uint32_t *>(tiled + tiled_codes_at(g, t, c) + lane * 16 + j * 4);
        nib[e] = (w >> pos) & 0xF;
      }
      o[2 + jb] = (uint8_t)(nib[0] | (nib[1] << 4));
    }
  } else {
    uint8_t *o = blocks + idx * 34;
    o[0] = (uint8_t)(s & 0xFF);
    o[1] = (uint8_t)((s >> 8) & 0xFF);
    for (int e = 0; e < 32; e++) {
      const int k = b * 32 + e;
      const int step = k / 16, kk = k % 16;
      const int c = step / 2;
      const int jj = kk & 3, lane = (ri & 7) * 4 + kk / 4;
      const int j = (step % 2) * 2 + (jj >= 2 ? 1 : 0);
      const int byte = (ri >= 8 ? 2 : 0) + (jj & 1);
      o[2 + e] = tiled[tiled_codes_at(g, t, c) + lane * 16 + j * 4 + byte] ^ 0x80;
    }
  }
}

bool ggml_fmt(int fmt) {
  return fmt == VXB_Q4_0 || fmt == VXB_Q8_0 || fmt == VXB_Q4_1 || fmt == VXB_GGML_F16 || fmt == VXB_GGML_F32;
}

int check_fmt(vxb_ctx *ctx, int fmt, const char *who) {
  if (fmt != VXB_Q4_0 && fmt != VXB_Q8_0) return set_error(ctx, VXB_EINVAL, "%s: unknown block format %d", who, fmt);
  return VXB_OK;
}

}  // namespace

VXB_API size_t vxb_block_bytes(int fmt, size_t n) {
  if (fmt == VXB_Q4_0) return (n + 31) / 32 * 18;
  if (fmt == VXB_Q8_0) return (n + 31) / 32 * 34;
  if (fmt == VXB_Q4_1) return (n + 31) / 32 * 20;
  if (fmt == VXB_GGML_F16) return n * 2;
  if (fmt == VXB_GGML_F32) return n * 4;
  return 0;
}

VXB_API int vxb_pack_blocks_f64(int fmt, const double *w, size_t n, uint8_t *out) {
  if (check_fmt(nullptr, fmt, "vxb_pack_blocks_f64")) return VXB_EINVAL;
  if (n && (!w || !out)) return set_error(nullptr, VXB_EINVAL, "vxb_pack_blocks_f64: null argument");
  return pack_blocks_host(fmt, w, n, out);
}

VXB_API int vxb_pack_blocks_f32(int fmt, const float *w, size_t n, uint8_t *out) {
  if (check_fmt(nullptr, fmt, "vxb_pack_blocks_f32")) return VXB_EINVAL;
  if (n && (!w || !out)) return set_error(nullptr, VXB_EINVAL, "vxb_pack_blocks_f32: null argument");
  return pack_blocks_host(fmt, w, n, out);
}

VXB_API int vxb_unpack_blocks(int fmt, const uint8_t *blocks, size_t n, float *out) {
  if (!ggml_fmt(fmt)) return set_error(nullptr, VXB_EINVAL, "vxb_unpack_blocks: unknown block format %d", fmt);
  if (n && (!blocks || !out)) return set_error(nullptr, VXB_EINVAL, "vxb_unpack_blocks: null argument");
  if (fmt == VXB_Q4_1 || fmt == VXB_GGML_F16 || fmt == VXB_GGML_F32) {
    for (size_t i = 0; i < n; i++) {
      if (fmt == VXB_Q4_1) {
        const uint8_t *blk = blocks + (i / 32) * 20;
        const float d = host_ref_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        const float m = host_ref_f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
        const uint8_t byte = blk[4 + (i % 32) / 2];
        volatile float prod = (float)((i & 1) ? (byte >> 4) : (byte & 0xF)) * d;  // rounded before the add
        out[i] = prod + m;
      } else if (fmt == VXB_GGML_F16) {
        out[i] = host_ref_f16_to_f32((uint16_t)(blocks[2 * i] | (blocks[2 * i + 1] << 8)));
      } else {
        std::memcpy(out + i, blocks + 4 * i, 4);
      }
    }
    return VXB_OK;
  }
  for (size_t i = 0; i < n; i++) {
    size_t b = i / 32, e = i % 32;
    if (fmt == VXB_Q4_0) {
      const uint8_t *blk = blocks + b * 18;
      float d = host_ref_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
      uint8_t byte = blk[2 + e / 2];
      int nib = (e & 1) ? (byte >> 4) : (byte & 0xF);
      out[i] = (float)nib - 8.0f;
      out[i] = out[i] * d;
    } else {
      const uint8_t *blk = blocks + b * 34;
      float d = host_ref_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
      out[i] = (float)(int8_t)blk[2 + e] * d;
    }
  }
  return VXB_OK;
}

VXB_API int vxb_quantize_blocks(vxb_ctx *ctx, int fmt, const float *d_w, size_t n, uint8_t *d_blocks,
                                void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_quantize_blocks: null context");
  if (int rc = check_fmt(ctx, fmt, "vxb_quantize_blocks")) return rc;
  if (n == 0) return VXB_OK;
  if (!d_w || !d_blocks) return set_error(ctx, VXB_EINVAL, "vxb_quantize_blocks: null pointer");
  if (int rc = use_device(ctx)) return rc;
  const size_t nb = (n + 31) / 32;
  const unsigned grid = (unsigned)((nb + 7) / 8);
  quantize_blocks_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(d_w, n, d_blocks, fmt == VXB_Q4_0);
  return launch_check(ctx, "quantize_blocks_kernel");
}

VXB_API int vxb_dequantize_blocks(vxb_ctx *ctx, int fmt, const uint8_t *d_blocks, size_t n, float *d_out,
                                  void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_dequantize_blocks: null context");
  if (!ggml_fmt(fmt)) return set_error(ctx, VXB_EINVAL, "vxb_dequantize_blocks: unknown block format %d", fmt);
  if (n == 0) return VXB_OK;
  if (!d_blocks || !d_out) return set_error(ctx, VXB_EINVAL, "vxb_dequantize_blocks: null pointer");
  if (int rc = use_device(ctx)) return rc;
  if (fmt != VXB_Q4_0 && fmt != VXB_Q8_0) {
    dequantize_ggml_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(d_blocks, n, d_out, fmt);
    return launch_check(ctx, "dequantize_ggml_kernel");
  }
  dequantize_blocks_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(d_blocks, n, d_out,
                                                                                          fmt == VXB_Q4_0);
  return launch_check(ctx, "dequantize_blocks_kernel");
}

VXB_API size_t vxb_tiled_bytes(int fmt, int N, int K) {
  if ((fmt != VXB_Q4_0 && fmt != VXB_Q8_0) || N <= 0 || K <= 0 || K % 32) return 0;
  return tiled_geom(fmt, N, K).total_bytes;
}

VXB_API int vxb_tile_weights(vxb_ctx *ctx, int fmt, const uint8_t *d_blocks, int N, int K, void *d_tiled,
                             void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_tile_weights: null context");
  if (int rc = check_fmt(ctx, fmt, "vxb_tile_weights")) return rc;
  if (N <= 0 || K <= 0 || K % 32)
    return set_error(ctx, VXB_EINVAL, "vxb_tile_weights: need N > 0 and K a positive multiple of 32 (N=%d K=%d)", N, K);
  if (!d_blocks || !d_tiled) return set_error(ctx, VXB_EINVAL, "vxb_tile_weights: null pointer");
  if (((uintptr_t)d_tiled) % 256) return set_error(ctx, VXB_EINVAL, "vxb_tile_weights: tiled buffer must be 256-byte aligned");
  if (int rc = use_device(ctx)) return rc;
  if (int rc = vxb::tile_header(ctx, fmt, N, K, d_tiled, (cudaStream_t)stream)) return rc;
  return vxb::tile_part(ctx, fmt, d_blocks, N, K, 0, N, d_tiled, (cudaStream_t)stream);
}

namespace vxb {

int tile_header(vxb_ctx *ctx, int fmt, int N, int K, void *d_tiled, cudaStream_t st) {
  const TiledGeom g = tiled_geom(fmt, N, K);
  uint32_t *hdr = (uint32_t *)d_tiled;
  // padding rows of the last 128-row group stay zero (code 0, scale 0)
  VXB_CUDA_TRY(ctx, cudaMemsetAsync(hdr, 0, g.total_bytes, st));
  tile_header_kernel<<<1, 1, 0, st>>>(hdr, fmt, N, K);
  return launch_check(ctx, "tile_header_kernel");
}

int tile_part(vxb_ctx *ctx, int fmt, const uint8_t *d_blocks, int nrows, int K, int row0, int N_total, void *d_tiled,
              cudaStream_t st) {
  if (row0 % 16 || (nrows % 16 && row0 + nrows != N_total) || row0 + nrows > N_total)
    return set_error(ctx, VXB_EINVAL, "tile_part: rows [%d, %d) of %d are not 16-row aligned", row0, row0 + nrows, N_total);
  const TiledGeom g = tiled_geom(fmt, N_total, K);
  uint8_t *base = (uint8_t *)d_tiled;
  const int ntiles = (nrows + 15) / 16;
  const size_t nc = (size_t)ntiles * g.n_chunks * 128, ns = (size_t)ntiles * g.n_blocks * 8;
  tile_codes_kernel<<<(unsigned)((nc + 255) / 256), 256, 0, st>>>(d_blocks, fmt, nrows, K, g, row0 / 16, base);
  if (int rc = launch_check(ctx, "tile_codes_kernel")) return rc;
  tile_scales_kernel<<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(d_blocks, fmt, nrows, K, g, row0 / 16, base);
  return launch_check(ctx, "tile_scales_kernel");
}

}  // namespace vxb

VXB_API int vxb_untile_weights(vxb_ctx *ctx, int fmt, const void *d_tiled, int N, int K, uint8_t *d_blocks,
                               void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_untile_weights: null context");
  if (int rc = check_fmt(ctx, fmt, "vxb_untile_weights")) return rc;
  if (N <= 0 || K <= 0 || K % 32) return set_error(ctx, VXB_EINVAL, "vxb_untile_weights: bad shape N=%d K=%d", N, K);
  if (!d_blocks || !d_tiled) return set_error(ctx, VXB_EINVAL, "vxb_untile_weights: null pointer");
  if (int rc = use_device(ctx)) return rc;
  TiledGeom g = tiled_geom(fmt, N, K);
  size_t n = (size_t)N * (K / 32);
  untile_kernel<<<(unsigned)((n + 127) / 128), 128, 0, (cudaStream_t)stream>>>((const uint8_t *)d_tiled, fmt, N, K,
                                                                              g, d_blocks);
  return launch_check(ctx, "untile_kernel");
}
