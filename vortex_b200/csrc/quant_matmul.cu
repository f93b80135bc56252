// Mean-scale quantized matrix multiply and the QuantTensor quantizer.
//
// Replaces QuantTensor::matmul for INT8 x INT8 and INT4 x INT4
// (src/quantize.rs:447-515, reached from the quantized_matmul builtin,
// src/interpreter.rs:7330-7346):
//
//   C[i, j] = (f64)(sum_p (A[i, p] - za) (B[p, j] - zb)) * a_scale * b_scale
//
// A [M, K] and B [K, N] are row-major code buffers (INT8: one two's-
// complement byte per element; INT4: two per byte, the even flat index in
// the low nibble, pack_int4 at src/quantize.rs:664-672). The sum is an i32
// that wraps on overflow like the reference's release build, so the kernel
// accumulates in 32-bit integer arithmetic (dp4a: four signed byte products
// per instruction, modular) and applies the zero points afterwards through
//   sum (a - za)(b - zb) = sum ab - zb sum a - za sum b + K za zb  (mod 2^32),
// which is exact in the ring of 32-bit integers. The scales are the mean of
// the group scales (get_scale, src/quantize.rs:534-545) and multiply the
// converted sum left to right in f64, as the reference does.
//
// Work per launch: M N K multiply-adds on 1-byte (INT8) or half-byte (INT4)
// operands; the CTA tile is 64 x 64 outputs, k staged 64 at a time in shared
// memory (A row-major, B transposed so both operands are k-contiguous words).
#include <cmath>
#include <cstring>

#include "vxb_internal.h"

using namespace vxb;

namespace {

constexpr int QM_TILE = 64;   // rows and columns of a CTA tile
constexpr int QM_BK = 64;     // k per stage
constexpr int QM_PAD = 4;     // bytes of padding per shared-memory row
constexpr int QM_THREADS = 256;

// element e of a code buffer as a signed integer
template <bool INT4>
__device__ __forceinline__ int code_at(const uint8_t *__restrict__ p, size_t e) {
  if (!INT4) return (int)(int8_t)__ldg(p + e);
  const int byte = __ldg(p + (e >> 1));
  const int nib = (e & 1) ? (byte >> 4) : (byte & 0xF);
  return (nib ^ 8) - 8;  // sign extension of the nibble
}

template <bool INT4>
__global__ void __launch_bounds__(QM_THREADS) quant_matmul_kernel(const uint8_t *__restrict__ A,
                                                                  const uint8_t *__restrict__ B, int M, int K, int N,
                                                                  double a_scale, double b_scale, int za, int zb,
                                                                  double *__restrict__ C) {
  __shared__ __align__(16) int8_t As[QM_TILE][QM_BK + QM_PAD];  // [row][k]
  __shared__ __align__(16) int8_t Bt[QM_TILE][QM_BK + QM_PAD];  // [col][k]
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;  // outputs: rows ty + 16 r, columns tx + 16 c
  const int m0 = blockIdx.y * QM_TILE, n0 = blockIdx.x * QM_TILE;
  int acc[4][4] = {};
  int sa[4] = {}, sb[4] = {};
  for (int k0 = 0; k0 < K; k0 += QM_BK) {
    // A tile: 64 rows x 64 k; each thread fills 16 consecutive k of one row
    {
      const int r = tid / 4, kc = (tid % 4) * 16;
      const int gi = m0 + r;
#pragma unroll
      for (int u = 0; u < 16; u++) {
        const int gk = k0 + kc + u;
        As[r][kc + u] = (int8_t)((gi < M && gk < K) ? code_at<INT4>(A, (size_t)gi * K + gk) : 0);
      }
    }
    // B tile: 64 k x 64 columns, stored transposed; each thread reads 16
    // consecutive columns of one k row
    {
      const int kr = tid / 4, jc = (tid % 4) * 16;
      const int gk = k0 + kr;
#pragma unroll
      for (int u = 0; u < 16; u++) {
        const int gj = n0 + jc + u;
        Bt[jc + u][kr] = (int8_t)((gk < K && gj < N) ? code_at<INT4>(B, (size_t)gk * N + gj) : 0);
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < QM_BK; kk += 4) {
      int a4[4], b4[4];
#pragma unroll
      for (int r = 0; r < 4; r++) a4[r] = *reinterpret_cast<const int *>(&As[ty + 16 * r][kk]);
#pragma unroll
      for (int c = 0; c < 4; c++) b4[c] = *reinterpret_cast<const int *>(&Bt[tx + 16 * c][kk]);
#pragma unroll
      for (int r = 0; r < 4; r++) {
        sa[r] = __dp4a(a4[r], 0x01010101, sa[r]);
#pragma unroll
        for (int c = 0; c < 4; c++) acc[r][c] = __dp4a(a4[r], b4[c], acc[r][c]);
      }
#pragma unroll
      for (int c = 0; c < 4; c++) sb[c] = __dp4a(0x01010101, b4[c], sb[c]);
    }
    __syncthreads();
  }
  const uint32_t kzz = (uint32_t)K * (uint32_t)za * (uint32_t)zb;
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int i = m0 + ty + 16 * r;
    if (i >= M) continue;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int j = n0 + tx + 16 * c;
      if (j >= N) continue;
      const uint32_t s = (uint32_t)acc[r][c] - (uint32_t)zb * (uint32_t)sa[r] - (uint32_t)za * (uint32_t)sb[c] + kzz;
      const double v = (double)(int32_t)s * a_scale;
      C[(size_t)i * N + j] = v * b_scale;
    }
  }
}

// ---------------- host quantizer (QuantTensor::quantize, INT8 / INT4) ----------------

int qt_code(double v, double scale, int qmin, int qmax) {
  if (scale == 0.0) return 0;
  const double r = std::round(v / scale);
  if (std::isnan(r)) return 0;  // `as i64` of NaN is 0
  if (r < qmin) return qmin;
  if (r > qmax) return qmax;
  return (int)r;
}

}  // namespace

VXB_API size_t vxb_qt_data_bytes(int fmt, size_t n) {
  if (fmt == VXB_QT_INT8) return n;
  if (fmt == VXB_QT_INT4) return (n + 1) / 2;
  return 0;
}

VXB_API size_t vxb_qt_num_groups(size_t n, size_t group_size) {
  if (group_size == 0) return 1;
  return n == 0 ? 0 : (n + group_size - 1) / group_size;
}

VXB_API int vxb_qt_quantize(int fmt, const double *h_data, size_t n, size_t group_size, uint8_t *h_packed,
                            double *h_scales, int64_t *h_zero_points) {
  if (fmt != VXB_QT_INT8 && fmt != VXB_QT_INT4)
    return set_error(nullptr, VXB_EINVAL, "vxb_qt_quantize: format %d (INT8 = 0, INT4 = 1)", fmt);
  if ((n && (!h_data || !h_packed)) || !h_scales || !h_zero_points)
    return set_error(nullptr, VXB_EINVAL, "vxb_qt_quantize: null argument");
  const int qmin = fmt == VXB_QT_INT8 ? -128 : -8, qmax = fmt == VXB_QT_INT8 ? 127 : 7;
  // calibrate_minmax (INT8: absmax / 127) and calibrate_minmax_range (INT4:
  // absmax / max(|-8|, |7|)); an empty or all-zero slice gives (1.0, 0)
  const double div = fmt == VXB_QT_INT8 ? 127.0 : 8.0;
  const size_t gs = group_size ? group_size : (n ? n : 1);
  if (n == 0) {
    h_scales[0] = 1.0;
    h_zero_points[0] = 0;
    return VXB_OK;
  }
  if (fmt == VXB_QT_INT4) std::memset(h_packed, 0, (n + 1) / 2);
  size_t g = 0;
  for (size_t s = 0; s < n; s += gs, g++) {
    const size_t len = s + gs <= n ? gs : n - s;
    double amax = 0.0;
    for (size_t i = 0; i < len; i++) amax = std::fmax(amax, std::fabs(h_data[s + i]));
    const double scale = amax == 0.0 ? 1.0 : amax / div;
    h_scales[g] = scale;
    h_zero_points[g] = 0;
    for (size_t i = 0; i < len; i++) {
      const int q = qt_code(h_data[s + i], scale, qmin, qmax);
      const size_t e = s + i;
      if (fmt == VXB_QT_INT8) {
        h_packed[e] = (uint8_t)(int8_t)q;
      } else {
        const uint8_t nib = (uint8_t)(q & 0xF);
        h_packed[e / 2] |= (e & 1) ? (uint8_t)(nib << 4) : nib;
      }
    }
  }
  return VXB_OK;
}

VXB_API int vxb_qt_mean_scale(const double *h_scales, size_t n_scales, double *out) {
  if (!out || (n_scales && !h_scales)) return set_error(nullptr, VXB_EINVAL, "vxb_qt_mean_scale: null argument");
  if (n_scales == 0) {
    *out = 1.0;
    return VXB_OK;
  }
  double s = 0.0;  // in order, as iter().sum()
  for (size_t i = 0; i < n_scales; i++) s += h_scales[i];
  *out = s / (double)n_scales;
  return VXB_OK;
}

VXB_API int vxb_quant_matmul(vxb_ctx *ctx, int fmt, const uint8_t *d_a, const uint8_t *d_b, int M, int K, int N,
                             double a_scale, double b_scale, int64_t a_zero_point, int64_t b_zero_point,
                             double *d_out, void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_quant_matmul: null context");
  if (fmt != VXB_QT_INT8 && fmt != VXB_QT_INT4)
    return set_error(ctx, VXB_EUNSUPPORTED, "vxb_quant_matmul: format %d (INT8 = 0 and INT4 = 1 are supported)", fmt);
  if (M < 0 || K < 0 || N < 0) return set_error(ctx, VXB_EINVAL, "vxb_quant_matmul: bad shape M=%d K=%d N=%d", M, K, N);
  if (M == 0 || N == 0) return VXB_OK;
  if (!d_a || !d_b || !d_out) return set_error(ctx, VXB_EINVAL, "vxb_quant_matmul: null pointer");
  if (int rc = use_device(ctx)) return rc;
  const dim3 grid((N + QM_TILE - 1) / QM_TILE, (M + QM_TILE - 1) / QM_TILE);
  // `zero_point as i32` in the reference: the low 32 bits
  const int za = (int)(uint32_t)(uint64_t)a_zero_point, zb = (int)(uint32_t)(uint64_t)b_zero_point;
  cudaStream_t st = (cudaStream_t)stream;
  if (fmt == VXB_QT_INT8)
    quant_matmul_kernel<false><<<grid, QM_THREADS, 0, st>>>(d_a, d_b, M, K, N, a_scale, b_scale, za, zb, d_out);
  else
    quant_matmul_kernel<true><<<grid, QM_THREADS, 0, st>>>(d_a, d_b, M, K, N, a_scale, b_scale, za, zb, d_out);
  return launch_check(ctx, "quant_matmul_kernel");
}
