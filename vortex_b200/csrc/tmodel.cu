// The reference's f32 GPT-style TransformerModel on the GPU
// (src/transformer.rs:15-841): token embedding + sinusoidal positions,
// pre-norm layers (LayerNorm eps 1e-5, multi-head attention with biased
// projections and an optional [S, S] mask, GELU feed-forward), final
// LayerNorm and output projection; Xavier initialisation from the
// reference's xorshift generator (seed 42).
//
// Every matrix product sums over its inner dimension in the reference's order
// with separately rounded multiplies and adds (no fused multiply-add), the
// bias and residual adds are separate, and LayerNorm's mean and variance are
// sequential sums, so linears, norms and score products reproduce the
// reference's f32 bits; exp / tanh come from the CUDA math library, within
// a few ulp of the host library's.
#include <cmath>
#include <vector>

#include "vxb_internal.h"

using namespace vxb;

struct vxb_tmodel {
  vxb_ctx *ctx = nullptr;
  vxb_tmodel_config cfg{};
  size_t n_params = 0;
  float *params = nullptr;  // device, params_vec order
  float *pe = nullptr;      // [max_seq, d] positional encoding
  cudaStream_t stream = nullptr;
};

namespace {

// params_vec layout sizes (src/transformer.rs: Linear::params_vec = weight
// [out, in] then bias [out]; layer = wq wk wv wo linear1 linear2 norm1 norm2)
size_t layer_params(const vxb_tmodel_config &c) {
  const size_t d = c.d_model, f = c.d_ff;
  return 4 * (d * d + d) + (f * d + f) + (d * f + d) + 4 * d;
}

size_t param_count(const vxb_tmodel_config &c) {
  const size_t d = c.d_model, V = c.vocab_size;
  return V * d + (size_t)c.n_layers * layer_params(c) + 2 * d + V * d + V;
}

// SimpleRng (src/transformer.rs:15-45): xorshift64 from seed + 1
struct XorShift {
  uint64_t s;
  explicit XorShift(uint64_t seed) : s(seed + 1) {}
  uint64_t next() {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return s;
  }
  float next_f32() {
    const float u = (float)(next() >> 40) / (float)(1ull << 24);
    return u * 2.0f - 1.0f;
  }
  float xavier(size_t fan_in, size_t fan_out) { return next_f32() * std::sqrt(6.0f / (float)(fan_in + fan_out)); }
};

void init_linear(XorShift &r, size_t in, size_t out, float *p) {
  for (size_t i = 0; i < out * in; i++) p[i] = r.xavier(in, out);
  for (size_t i = 0; i < out; i++) p[out * in + i] = 0.0f;
}

// TransformerModel::new: embedding, then per layer wq wk wv wo linear1
// linear2 (norms gamma 1, beta 0), final norm, output projection
void init_params(const vxb_tmodel_config &c, std::vector<float> &p) {
  p.assign(param_count(c), 0.f);
  XorShift r(42);
  const size_t d = c.d_model, f = c.d_ff, V = c.vocab_size;
  float *q = p.data();
  for (size_t i = 0; i < V * d; i++) q[i] = r.xavier(V, d);
  q += V * d;
  for (int l = 0; l < c.n_layers; l++) {
    for (int m = 0; m < 4; m++, q += d * d + d) init_linear(r, d, d, q);
    init_linear(r, d, f, q);
    q += f * d + f;
    init_linear(r, f, d, q);
    q += d * f + d;
    for (int m = 0; m < 2; m++, q += 2 * d)
      for (size_t i = 0; i < d; i++) q[i] = 1.0f;
  }
  for (size_t i = 0; i < d; i++) q[i] = 1.0f;
  q += 2 * d;
  init_linear(r, d, V, q);
}

// make_pos_encoding (src/transformer.rs:655-670), on the host
void pos_encoding(int max_len, int d, std::vector<float> &out) {
  out.resize((size_t)max_len * d);
  for (int pos = 0; pos < max_len; pos++)
    for (int i = 0; i < d; i++) {
      const float angle = (float)pos / std::pow(10000.0f, (float)(2 * (i / 2)) / (float)d);
      out[(size_t)pos * d + i] = (i % 2 == 0) ? std::sin(angle) : std::cos(angle);
    }
}

__global__ void embed_pe_kernel(const float *__restrict__ emb, const float *__restrict__ pe,
                                const int32_t *__restrict__ tok, int d, float *__restrict__ x) {
  const int i = blockIdx.x;
  for (int j = threadIdx.x; j < d; j += blockDim.x) x[(size_t)i * d + j] = emb[(size_t)tok[i] * d + j] + pe[(size_t)i * d + j];
}

// y[m, n] = sum_k x[m, k] * w[n, k] (+ b[n]); every output sums k in order
// with rounded multiply and add; 64x64 tile, 16x16 threads, 4x4 each
constexpr int LT = 64, LK = 16;
__global__ void linear_kernel(const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ b,
                              int M, int N, int K, float *__restrict__ y) {
  __shared__ float xs[LK][LT + 1], ws[LK][LT + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * LT, n0 = blockIdx.x * LT;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += LK) {
    for (int i = threadIdx.x; i < LT * LK; i += 256) {
      const int r = i / LK, k = i % LK;
      xs[k][r] = (m0 + r < M && k0 + k < K) ? x[(size_t)(m0 + r) * K + k0 + k] : 0.f;
      ws[k][r] = (n0 + r < N && k0 + k < K) ? w[(size_t)(n0 + r) * K + k0 + k] : 0.f;
    }
    __syncthreads();
    const int kmax = min(LK, K - k0);
    for (int k = 0; k < kmax; k++) {
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int c = 0; c < 4; c++) acc[a][c] = __fadd_rn(acc[a][c], __fmul_rn(xs[k][ty * 4 + a], ws[k][tx * 4 + c]));
    }
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int m = m0 + ty * 4 + a, n = n0 + tx * 4 + c;
      if (m < M && n < N) y[(size_t)m * N + n] = b ? __fadd_rn(acc[a][c], b[n]) : acc[a][c];
    }
}

// LayerNorm::forward: one block per row; mean and variance summed in order by
// one thread, then every element normalised in parallel
__global__ void layernorm_kernel(const float *__restrict__ x, int d, const float *__restrict__ g,
                                 const float *__restrict__ b, float eps, float *__restrict__ y) {
  __shared__ float s_mean, s_inv;
  const float *row = x + (size_t)blockIdx.x * d;
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int j = 0; j < d; j++) s = __fadd_rn(s, row[j]);
    const float mean = __fdiv_rn(s, (float)d);
    float v = 0.f;
    for (int j = 0; j < d; j++) {
      const float t = __fsub_rn(row[j], mean);
      v = __fadd_rn(v, __fmul_rn(t, t));
    }
    s_mean = mean;
    s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, (float)d), eps)));
  }
  __syncthreads();
  for (int j = threadIdx.x; j < d; j += blockDim.x)
    y[(size_t)blockIdx.x * d + j] =
        __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(row[j], s_mean), s_inv), g[j]), b[j]);
}

__global__ void gelu_kernel(const float *__restrict__ x, size_t n, float *__restrict__ y) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float sqrt_2_pi = __fsqrt_rn(__fdiv_rn(2.0f, 3.14159265358979323846f));
  const float v = x[i];
  const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
  const float inner = __fmul_rn(sqrt_2_pi, __fadd_rn(v, cube));
  y[i] = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(inner)));
}

__global__ void add_kernel(float *__restrict__ x, const float *__restrict__ a, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __fadd_rn(x[i], a[i]);
}

// scaled dot-product attention of one head and one query row per block:
// scores in order over the head dim, scaled, masked (< 0.5 -> -1e9), softmax
// (max, exp, sequential sum, divide), then P V summed in key order
__global__ void attention_kernel(const float *__restrict__ qkv_q, const float *__restrict__ qkv_k,
                                 const float *__restrict__ qkv_v, const float *__restrict__ mask, int S, int d,
                                 int hd, float scale, float *__restrict__ out) {
  extern __shared__ float p[];  // [S]
  const int i = blockIdx.x, h = blockIdx.y;
  const float *q = qkv_q + (size_t)i * d + h * hd;
  for (int j = threadIdx.x; j < S; j += blockDim.x) {
    const float *k = qkv_k + (size_t)j * d + h * hd;
    float s = 0.f;
    for (int t = 0; t < hd; t++) s = __fadd_rn(s, __fmul_rn(q[t], k[t]));
    float sv = __fmul_rn(s, scale);
    if (mask && mask[(size_t)i * S + j] < 0.5f) sv = -1e9f;
    p[j] = sv;
  }
  __syncthreads();
  __shared__ float s_max, s_sum;
  if (threadIdx.x == 0) {
    float mx = -INFINITY;
    for (int j = 0; j < S; j++) mx = fmaxf(mx, p[j]);
    float sum = 0.f;
    for (int j = 0; j < S; j++) {
      const float e = expf(__fsub_rn(p[j], mx));
      p[j] = e;
      sum = __fadd_rn(sum, e);
    }
    s_max = mx;
    s_sum = sum;
  }
  __syncthreads();
  if (s_sum > 0.f)
    for (int j = threadIdx.x; j < S; j += blockDim.x) p[j] = __fdiv_rn(p[j], s_sum);
  __syncthreads();
  for (int t = threadIdx.x; t < hd; t += blockDim.x) {
    float s = 0.f;
    for (int j = 0; j < S; j++) s = __fadd_rn(s, __fmul_rn(p[j], qkv_v[(size_t)j * d + h * hd + t]));
    out[(size_t)i * d + h * hd + t] = s;
  }
}

int linear(vxb_tmodel *m, const float *x, int M, const float *w, const float *b, int in, int out, float *y) {
  dim3 grid((out + LT - 1) / LT, (M + LT - 1) / LT);
  linear_kernel<<<grid, 256, 0, m->stream>>>(x, w, b, M, out, in, y);
  return launch_check(m->ctx, "linear_kernel");
}

}  // namespace

VXB_API int vxb_tmodel_create(vxb_ctx *ctx, const vxb_tmodel_config *cfg, vxb_tmodel **out) {
  if (!ctx || !cfg || !out) return set_error(ctx, VXB_EINVAL, "vxb_tmodel_create: null argument");
  *out = nullptr;
  const vxb_tmodel_config &c = *cfg;
  if (c.vocab_size <= 0 || c.d_model <= 0 || c.n_heads <= 0 || c.n_layers < 0 || c.d_ff <= 0 || c.max_seq_len <= 0 ||
      c.d_model % c.n_heads)
    return set_error(ctx, VXB_EINVAL, "vxb_tmodel_create: bad configuration (d_model must be divisible by n_heads)");
  if (int rc = use_device(ctx)) return rc;
  vxb_tmodel *m = new vxb_tmodel();
  m->ctx = ctx;
  m->cfg = c;
  m->n_params = param_count(c);
  std::vector<float> p, pe;
  init_params(c, p);
  pos_encoding(c.max_seq_len, c.d_model, pe);
  int rc = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) == cudaSuccess ? VXB_OK : VXB_ECUDA;
  if (!rc && (cudaMalloc(&m->params, m->n_params * 4) != cudaSuccess || cudaMalloc(&m->pe, pe.size() * 4) != cudaSuccess))
    rc = set_error(ctx, VXB_ENOMEM, "vxb_tmodel_create: parameter allocation");
  if (!rc && (cudaMemcpy(m->params, p.data(), m->n_params * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
              cudaMemcpy(m->pe, pe.data(), pe.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess))
    rc = set_error(ctx, VXB_ECUDA, "vxb_tmodel_create: parameter upload");
  if (rc) {
    cudaGetLastError();
    vxb_tmodel_destroy(m);
    return rc;
  }
  *out = m;
  return VXB_OK;
}

VXB_API int vxb_tmodel_destroy(vxb_tmodel *m) {
  if (!m) return VXB_OK;
  use_device(m->ctx);
  if (m->params) cudaFree(m->params);
  if (m->pe) cudaFree(m->pe);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
  return VXB_OK;
}

VXB_API int vxb_tmodel_param_count(const vxb_tmodel *m, size_t *n) {
  if (!m || !n) return set_error(nullptr, VXB_EINVAL, "vxb_tmodel_param_count: null argument");
  *n = m->n_params;
  return VXB_OK;
}

VXB_API int vxb_tmodel_set_params(vxb_tmodel *m, const float *h_params, size_t n) {
  if (!m || !h_params) return set_error(m ? m->ctx : nullptr, VXB_EINVAL, "vxb_tmodel_set_params: null argument");
  if (n != m->n_params) return set_error(m->ctx, VXB_EINVAL, "vxb_tmodel_set_params: %zu values, expected %zu", n, m->n_params);
  if (int rc = use_device(m->ctx)) return rc;
  VXB_CUDA_TRY(m->ctx, cudaMemcpy(m->params, h_params, n * 4, cudaMemcpyHostToDevice));
  return VXB_OK;
}

VXB_API int vxb_tmodel_get_params(vxb_tmodel *m, float *h_params, size_t n) {
  if (!m || !h_params) return set_error(m ? m->ctx : nullptr, VXB_EINVAL, "vxb_tmodel_get_params: null argument");
  if (n != m->n_params) return set_error(m->ctx, VXB_EINVAL, "vxb_tmodel_get_params: %zu values, expected %zu", n, m->n_params);
  if (int rc = use_device(m->ctx)) return rc;
  VXB_CUDA_TRY(m->ctx, cudaMemcpy(h_params, m->params, n * 4, cudaMemcpyDeviceToHost));
  return VXB_OK;
}

VXB_API int vxb_tmodel_forward(vxb_tmodel *m, const int32_t *h_tokens, int S, const float *h_mask, float *h_logits) {
  if (!m || !h_tokens || !h_logits) return set_error(m ? m->ctx : nullptr, VXB_EINVAL, "vxb_tmodel_forward: null argument");
  const vxb_tmodel_config &c = m->cfg;
  vxb_ctx *ctx = m->ctx;
  if (S < 1 || S > c.max_seq_len) return set_error(ctx, VXB_EINVAL, "vxb_tmodel_forward: %d tokens (1..%d)", S, c.max_seq_len);
  for (int i = 0; i < S; i++)
    if (h_tokens[i] < 0 || h_tokens[i] >= c.vocab_size)
      return set_error(ctx, VXB_EINVAL, "vxb_tmodel_forward: token id out of range");
  if (int rc = use_device(ctx)) return rc;
  const size_t d = c.d_model, f = c.d_ff, V = c.vocab_size;
  const int H = c.n_heads, hd = c.d_model / c.n_heads;
  // activations: x, n, q, k, v, a, merged [S, d]; hid, act [S, f]; logits [S, V]; tokens; mask
  const size_t fl = (size_t)S * (7 * d + 2 * f + V) + (h_mask ? (size_t)S * S : 0);
  float *buf = nullptr;
  int32_t *tok = nullptr;
  if (cudaMalloc(&buf, fl * 4) != cudaSuccess || cudaMalloc(&tok, S * 4) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(buf);
    return set_error(ctx, VXB_ENOMEM, "vxb_tmodel_forward: activation allocation");
  }
  float *x = buf, *nrm = x + S * d, *q = nrm + S * d, *k = q + S * d, *v = k + S * d, *a = v + S * d, *mg = a + S * d;
  float *hid = mg + S * d, *act = hid + S * f, *logits = act + S * f, *mask = h_mask ? logits + S * V : nullptr;
  cudaStream_t st = m->stream;
  int rc = VXB_OK;
  if (cudaMemcpyAsync(tok, h_tokens, S * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      (h_mask && cudaMemcpyAsync(mask, h_mask, (size_t)S * S * 4, cudaMemcpyHostToDevice, st) != cudaSuccess))
    rc = set_error(ctx, VXB_ECUDA, "vxb_tmodel_forward: upload");
  if (!rc) {
    embed_pe_kernel<<<S, 256, 0, st>>>(m->params, m->pe, tok, (int)d, x);
    rc = launch_check(ctx, "embed_pe_kernel");
  }
  const float *p = m->params + V * d;
  const float scale = 1.0f / std::sqrt((float)hd);
  for (int l = 0; l < c.n_layers && !rc; l++) {
    const float *wq = p, *wk = wq + d * d + d, *wv = wk + d * d + d, *wo = wv + d * d + d;
    const float *l1 = wo + d * d + d, *l2 = l1 + f * d + f, *n1 = l2 + d * f + d, *n2 = n1 + 2 * d;
    layernorm_kernel<<<S, 128, 0, st>>>(x, (int)d, n1, n1 + d, 1e-5f, nrm);
    rc = launch_check(ctx, "layernorm_kernel");
    if (!rc) rc = linear(m, nrm, S, wq, wq + d * d, (int)d, (int)d, q);
    if (!rc) rc = linear(m, nrm, S, wk, wk + d * d, (int)d, (int)d, k);
    if (!rc) rc = linear(m, nrm, S, wv, wv + d * d, (int)d, (int)d, v);
    if (!rc) {
      attention_kernel<<<dim3(S, H), 128, S * 4, st>>>(q, k, v, mask, S, (int)d, hd, scale, mg);
      rc = launch_check(ctx, "attention_kernel");
    }
    if (!rc) rc = linear(m, mg, S, wo, wo + d * d, (int)d, (int)d, a);
    if (!rc) {
      add_kernel<<<(unsigned)((S * d + 255) / 256), 256, 0, st>>>(x, a, S * d);
      layernorm_kernel<<<S, 128, 0, st>>>(x, (int)d, n2, n2 + d, 1e-5f, nrm);
      rc = launch_check(ctx, "layernorm_kernel");
    }
    if (!rc) rc = linear(m, nrm, S, l1, l1 + f * d, (int)d, (int)f, hid);
    if (!rc) {
      gelu_kernel<<<(unsigned)((S * f + 255) / 256), 256, 0, st>>>(hid, S * f, act);
      rc = launch_check(ctx, "gelu_kernel");
    }
    if (!rc) rc = linear(m, act, S, l2, l2 + d * f, (int)f, (int)d, a);
    if (!rc) {
      add_kernel<<<(unsigned)((S * d + 255) / 256), 256, 0, st>>>(x, a, S * d);
      rc = launch_check(ctx, "add_kernel");
    }
    p += layer_params(c);
  }
  if (!rc) {
    layernorm_kernel<<<S, 128, 0, st>>>(x, (int)d, p, p + d, 1e-5f, nrm);
    rc = launch_check(ctx, "layernorm_kernel");
  }
  p += 2 * d;
  if (!rc) rc = linear(m, nrm, S, p, p + V * d, (int)d, (int)V, logits);
  if (!rc && cudaMemcpyAsync(h_logits, logits, (size_t)S * V * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    rc = set_error(ctx, VXB_ECUDA, "vxb_tmodel_forward: download");
  if (cudaStreamSynchronize(st) != cudaSuccess && !rc) rc = set_error(ctx, VXB_ECUDA, "vxb_tmodel_forward: sync");
  cudaFree(buf);
  cudaFree(tok);
  return rc;
}
