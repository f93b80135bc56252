// Nucleus (top-p) sampling on the device, bit-matched to the reference's
// sample_top_p (stdlib/ai/transformer.vx:1179-1260), and the continuous-
// batching slot table (ContinuousBatcher, src/kv_cache.rs:117-154).
//
// sample_top_p computes everything in f64 in a fixed order: scaled = logit /
// temperature, mx = max, e = _exp(scaled - mx) with the file's own series
// exponential (36-80), psum = sum of e in index order, p = e / psum; the
// indices are exchange-sorted by descending p; cumsum in that order until it
// reaches top_p gives the cutoff; u = LCG(seed) / 2^31; the first position
// whose running sum of p / renorm reaches u is returned (index 0 of the
// order if none). Per row (one CTA each):
//   1. topp_probs_kernel: the element-wise steps in parallel, the two ordered
//      sums by one thread (a rounded sequential sum has no parallel form);
//   2. a stable descending segmented sort of (p, index): the sorted values
//      are those of the exchange sort, and so are the cumulative sums (equal
//      values added in either order give the same bits);
//   3. topp_select_kernel: the cutoff and draw scans by one thread. When the
//      selected value is unique its index is the answer. When it is tied, the
//      order inside the tie group is the exchange sort's own (not stable), so
//      the kernel replays the exchange sort, restricted to the entries with
//      p >= that value (their final order depends on nothing else), up to the
//      selected position: each pass of the sort moves the strict prefix
//      maxima of the remaining entries one maximum to the right and the last
//      one to the front, which a CTA applies with two block scans per pass.
#include <cub/device/device_segmented_sort.cuh>

#include <cmath>
#include <vector>

#include "vxb_internal.h"

using namespace vxb;

namespace {

constexpr int TP_THREADS = 1024;
constexpr int TP_MAX_CHUNK = 128;  // replay: entries per thread, vocab <= 131072

// _exp of stdlib/ai/transformer.vx:36-80 with every f64 operation rounded on
// its own (no contraction), as the interpreter evaluates it.
__device__ double vx_exp(double x) {
  if (x > 88.0) return 1.0e38;
  if (x < -88.0) return 0.0;
  const double ln2 = 0.6931471805599453;
  const double k_f = __ddiv_rn(x, ln2);
  const long long k = k_f >= 0.0 ? (long long)__dadd_rn(k_f, 0.5) : (long long)__dadd_rn(k_f, -0.5);
  const double r = __dadd_rn(x, -__dmul_rn((double)k, ln2));
  double sum = 1.0, term = 1.0;
#pragma unroll
  for (int i = 1; i <= 20; i++) {
    term = __ddiv_rn(__dmul_rn(term, r), (double)i);
    sum = __dadd_rn(sum, term);
  }
  double pow2 = 1.0;
  if (k >= 0) {
    for (long long j = 0; j < k; j++) pow2 = __dmul_rn(pow2, 2.0);
  } else {
    for (long long j = 0; j < -k; j++) pow2 = __ddiv_rn(pow2, 2.0);
  }
  return __dmul_rn(sum, pow2);
}

template <typename T, typename Op>
__device__ T block_reduce(T v, Op op, T ident, T *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    T w = lane < (int)(blockDim.x >> 5) ? red[lane] : ident;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = op(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (lane == 0) red[0] = w;
  }
  __syncthreads();
  return red[0];
}

// exclusive scan with `op` over the threads of the block (thread order)
template <typename T, typename Op>
__device__ T block_excl_scan(T v, Op op, T ident, T *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl = op(incl, t);
  }
  __syncthreads();
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    T w = lane < (int)(blockDim.x >> 5) ? red[lane] : ident;
    T wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi = op(wi, t);
    }
    red[lane] = wi;  // inclusive over warps
  }
  __syncthreads();
  T excl = __shfl_up_sync(0xffffffffu, incl, 1);
  if (lane == 0) excl = ident;
  if (warp > 0) excl = lane == 0 ? red[warp - 1] : op(red[warp - 1], excl);
  return excl;
}

struct MaxD {
  __device__ double operator()(double a, double b) const { return a > b ? a : b; }
};
struct MaxI {
  __device__ int operator()(int a, int b) const { return a > b ? a : b; }
};
struct AddI {
  __device__ int operator()(int a, int b) const { return a + b; }
};

// probs[r, i] = e_i / psum, idx[r, i] = i
__global__ void __launch_bounds__(TP_THREADS) topp_probs_kernel(const float *__restrict__ logits, int vocab,
                                                                 double temperature, double *__restrict__ probs,
                                                                 int *__restrict__ idx) {
  __shared__ double red[32];
  __shared__ double s_psum;
  const int row = blockIdx.x;
  const float *lg = logits + (size_t)row * vocab;
  double *p = probs + (size_t)row * vocab;
  int *ix = idx + (size_t)row * vocab;
  double mx = -INFINITY;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) mx = fmax(mx, __ddiv_rn((double)lg[i], temperature));
  mx = block_reduce<double>(mx, MaxD(), -INFINITY, red);
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
    p[i] = vx_exp(__dadd_rn(__ddiv_rn((double)lg[i], temperature), -mx));
    ix[i] = i;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;  // in index order
    for (int i = 0; i < vocab; i++) s = __dadd_rn(s, p[i]);
    s_psum = s;
  }
  __syncthreads();
  const double psum = s_psum;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) p[i] = __ddiv_rn(p[i], psum);
}

// cutoff, draw and the answer (with the exchange-sort replay for ties)
__global__ void __launch_bounds__(TP_THREADS) topp_select_kernel(
    const double *__restrict__ probs, const double *__restrict__ sorted_p, const int *__restrict__ sorted_i,
    const double *__restrict__ u_row, int vocab, double top_p, double *__restrict__ qbuf, int *__restrict__ cur_i,
    double *__restrict__ cur_v, int32_t *__restrict__ out) {
  __shared__ double s_renorm;
  __shared__ int s_cutoff, s_pos;
  __shared__ double redd[32];
  __shared__ int redi[32];
  const int row = blockIdx.x, tid = threadIdx.x;
  const double *p = probs + (size_t)row * vocab;
  const double *sp = sorted_p + (size_t)row * vocab;
  const int *si = sorted_i + (size_t)row * vocab;
  double *q = qbuf + (size_t)row * vocab;
  if (tid == 0) {
    double c = 0.0;
    int cutoff = vocab;
    for (int k = 0; k < vocab; k++) {
      c = __dadd_rn(c, sp[k]);
      if (c >= top_p) {
        cutoff = k + 1;
        break;
      }
    }
    s_cutoff = cutoff;
    s_renorm = c;  // the renormalising sum repeats the same additions
  }
  __syncthreads();
  const int cutoff = s_cutoff;
  const double renorm = s_renorm;
  for (int k = tid; k < cutoff; k += blockDim.x) q[k] = __ddiv_rn(sp[k], renorm);
  __syncthreads();
  if (tid == 0) {
    const double u = u_row[row];
    double acc = 0.0;
    int pos = -1;
    for (int k = 0; k < cutoff; k++) {
      acc = __dadd_rn(acc, q[k]);
      if (acc >= u) {
        pos = k;
        break;
      }
    }
    s_pos = pos;
  }
  __syncthreads();
  const int s = s_pos;
  if (s < 0) {  // no position reached u: index 0 of the order, the first maximum
    if (tid == 0) out[row] = si[0];
    return;
  }
  const double v = sp[s];
  const bool tied = (s > 0 && sp[s - 1] == v) || (s + 1 < vocab && sp[s + 1] == v);
  if (!tied) {
    if (tid == 0) out[row] = si[s];
    return;
  }
  // replay: the entries with p >= v in index order
  int *ci = cur_i + (size_t)row * vocab;
  double *cv = cur_v + (size_t)row * vocab;
  {
    const int chunk = (vocab + TP_THREADS - 1) / TP_THREADS;
    const int i0 = tid * chunk, i1 = min(vocab, i0 + chunk);
    int cnt = 0;
    for (int i = i0; i < i1; i++) cnt += p[i] >= v;
    int o = block_excl_scan(cnt, AddI(), 0, redi);
    for (int i = i0; i < i1; i++)
      if (p[i] >= v) {
        ci[o] = i;
        cv[o] = p[i];
        o++;
      }
  }
  __syncthreads();
  int m = 0;
  {
    int cnt = 0;
    for (int i = tid; i < vocab; i += blockDim.x) cnt += p[i] >= v;
    m = block_reduce(cnt, AddI(), 0, redi);
  }
  int rec[TP_MAX_CHUNK];
  int gi[TP_MAX_CHUNK];
  double gv[TP_MAX_CHUNK];
  for (int a = 0; a <= s && a < m - 1; a++) {
    const int n_act = m - a;
    const int chunk = (n_act + TP_THREADS - 1) / TP_THREADS;
    const int p0 = a + tid * chunk, p1 = min(m, p0 + chunk);
    double cmax = -INFINITY;
    for (int x = p0; x < p1; x++) cmax = fmax(cmax, cv[x]);
    const double before = block_excl_scan<double>(cmax, MaxD(), -INFINITY, redd);
    // strict prefix maxima: position a holds the running maximum first
    double run = before;
    int nrec = 0;
    for (int x = p0; x < p1; x++) {
      const double val = cv[x];
      if (x == a || val > run) {
        rec[nrec++] = x;
        run = val;
      }
    }
    const int last = nrec ? rec[nrec - 1] : -1;
    const int prev = block_excl_scan(last, MaxI(), -1, redi);
    const int rk = block_reduce(last, MaxI(), -1, redi);
    for (int r = 0; r < nrec; r++) {
      const int pred = rec[r] == a ? rk : (r == 0 ? prev : rec[r - 1]);
      gi[r] = ci[pred];
      gv[r] = cv[pred];
    }
    __syncthreads();
    for (int r = 0; r < nrec; r++) {
      ci[rec[r]] = gi[r];
      cv[rec[r]] = gv[r];
    }
    __syncthreads();
  }
  if (tid == 0) out[row] = ci[s];
}

// LCG draw of sample_top_p with the interpreter's 128-bit integers
double lcg_uniform(int64_t seed) {
  __int128 st = (__int128)1664525 * (__int128)seed + (__int128)1013904223;
  st = st % (__int128)2147483648LL;
  return (double)(int64_t)st / 2147483648.0;
}

}  // namespace

VXB_API int vxb_sample_top_p(vxb_ctx *ctx, const float *d_logits, int rows, int vocab, double temperature,
                             double top_p, const int64_t *h_seeds, int32_t *d_out, void *stream) {
  if (!ctx) return set_error(nullptr, VXB_EINVAL, "vxb_sample_top_p: null context");
  if (rows < 0 || vocab < 1 || vocab > TP_THREADS * TP_MAX_CHUNK)
    return set_error(ctx, VXB_EINVAL, "vxb_sample_top_p: rows %d, vocab %d (1..%d)", rows, vocab,
                     TP_THREADS * TP_MAX_CHUNK);
  if (rows == 0) return VXB_OK;
  if (!d_logits || !h_seeds || !d_out) return set_error(ctx, VXB_EINVAL, "vxb_sample_top_p: null pointer");
  if (int rc = use_device(ctx)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t n = (size_t)rows * vocab;
  // workspace: probs, sorted probs, q (f64); idx, sorted idx, replay idx (i32);
  // replay values (f64); offsets; draws; CUB temporary storage
  size_t cub_bytes = 0;
  cub::DeviceSegmentedSort::StableSortPairsDescending(nullptr, cub_bytes, (const double *)nullptr, (double *)nullptr,
                                                     (const int *)nullptr, (int *)nullptr, (int)n, rows,
                                                     (const int *)nullptr, (const int *)nullptr, st);
  auto al = [](size_t b) { return round_up(b, 256); };
  const size_t o_sp = al(n * 8), o_q = o_sp + al(n * 8), o_cv = o_q + al(n * 8), o_ix = o_cv + al(n * 8),
               o_si = o_ix + al(n * 4), o_ci = o_si + al(n * 4), o_off = o_ci + al(n * 4),
               o_u = o_off + al((size_t)(rows + 1) * 4), o_cub = o_u + al((size_t)rows * 8),
               total = o_cub + al(cub_bytes);
  if (int rc = ws_reserve(ctx, total, 0)) return rc;
  uint8_t *ws = (uint8_t *)ctx->ws;
  double *probs = (double *)ws, *sp = (double *)(ws + o_sp), *q = (double *)(ws + o_q), *cv = (double *)(ws + o_cv);
  int *ix = (int *)(ws + o_ix), *si = (int *)(ws + o_si), *ci = (int *)(ws + o_ci), *off = (int *)(ws + o_off);
  double *u = (double *)(ws + o_u);
  std::vector<int> h_off(rows + 1);
  for (int r = 0; r <= rows; r++) h_off[r] = r * vocab;
  std::vector<double> h_u(rows);
  for (int r = 0; r < rows; r++) h_u[r] = lcg_uniform(h_seeds[r]);
  VXB_CUDA_TRY(ctx, cudaMemcpyAsync(off, h_off.data(), (rows + 1) * sizeof(int), cudaMemcpyHostToDevice, st));
  VXB_CUDA_TRY(ctx, cudaMemcpyAsync(u, h_u.data(), rows * sizeof(double), cudaMemcpyHostToDevice, st));
  topp_probs_kernel<<<rows, TP_THREADS, 0, st>>>(d_logits, vocab, temperature, probs, ix);
  if (int rc = launch_check(ctx, "topp_probs_kernel")) return rc;
  size_t tb = cub_bytes;
  VXB_CUDA_TRY(ctx, cub::DeviceSegmentedSort::StableSortPairsDescending(ws + o_cub, tb, probs, sp, ix, si, (int)n,
                                                                      rows, off, off + 1, st));
  topp_select_kernel<<<rows, TP_THREADS, 0, st>>>(probs, sp, si, u, vocab, top_p, q, ci, cv, d_out);
  if (int rc = launch_check(ctx, "topp_select_kernel")) return rc;
  // the host vectors above must outlive the asynchronous copies
  VXB_CUDA_TRY(ctx, cudaStreamSynchronize(st));
  return VXB_OK;
}

// ---------------------------------------------------------------------------
// ContinuousBatcher (src/kv_cache.rs:117-154): a fixed number of slots; a
// request takes the lowest free slot and the next sequence id, removal frees
// the slot (the id is not reused).
// ---------------------------------------------------------------------------
struct vxb_batcher {
  struct Slot {
    bool used = false;
    int64_t seq_id = 0;
    std::vector<uint64_t> tokens;
    int64_t position = 0;
    bool is_prefill = true, is_done = false;
  };
  std::vector<Slot> slots;
  int64_t next_seq_id = 0;
};

VXB_API int vxb_batcher_create(int max_batch_size, vxb_batcher **out) {
  if (!out || max_batch_size < 0) return set_error(nullptr, VXB_EINVAL, "vxb_batcher_create: bad argument");
  vxb_batcher *b = new vxb_batcher();
  b->slots.resize(max_batch_size);
  *out = b;
  return VXB_OK;
}

VXB_API int vxb_batcher_destroy(vxb_batcher *b) {
  delete b;
  return VXB_OK;
}

VXB_API int vxb_batcher_add(vxb_batcher *b, const uint64_t *h_tokens, size_t n_tokens, int *slot_out) {
  if (!b || !slot_out || (n_tokens && !h_tokens)) return set_error(nullptr, VXB_EINVAL, "vxb_batcher_add: null argument");
  for (size_t i = 0; i < b->slots.size(); i++) {
    auto &s = b->slots[i];
    if (!s.used) {
      s.used = true;
      s.seq_id = b->next_seq_id++;
      s.tokens.assign(h_tokens, h_tokens + n_tokens);
      s.position = 0;
      s.is_prefill = true;
      s.is_done = false;
      *slot_out = (int)i;
      return VXB_OK;
    }
  }
  *slot_out = -1;
  return set_error(nullptr, VXB_ENOBLOCKS, "batcher full");  // the builtin's error (src/kv_cache.rs:266)
}

VXB_API int vxb_batcher_remove(vxb_batcher *b, int slot) {
  if (!b) return set_error(nullptr, VXB_EINVAL, "vxb_batcher_remove: null batcher");
  if (slot >= 0 && (size_t)slot < b->slots.size()) b->slots[slot] = vxb_batcher::Slot();
  return VXB_OK;
}

VXB_API int vxb_batcher_num_active(const vxb_batcher *b, int *out) {
  if (!b || !out) return set_error(nullptr, VXB_EINVAL, "vxb_batcher_num_active: null argument");
  int n = 0;
  for (const auto &s : b->slots) n += s.used;
  *out = n;
  return VXB_OK;
}

VXB_API int vxb_batcher_slot(const vxb_batcher *b, int slot, int64_t *seq_id, int64_t *position, int *is_prefill,
                             int *is_done, size_t *n_tokens) {
  if (!b) return set_error(nullptr, VXB_EINVAL, "vxb_batcher_slot: null batcher");
  if (slot < 0 || (size_t)slot >= b->slots.size() || !b->slots[slot].used)
    return set_error(nullptr, VXB_EINVAL, "vxb_batcher_slot: slot %d is empty", slot);
  const auto &s = b->slots[slot];
  if (seq_id) *seq_id = s.seq_id;
  if (position) *position = s.position;
  if (is_prefill) *is_prefill = s.is_prefill;
  if (is_done) *is_done = s.is_done;
  if (n_tokens) *n_tokens = s.tokens.size();
  return VXB_OK;
}

// Advance a slot after a step: `n` processed tokens (the prompt at prefill,
// then one per decode step), the prefill flag cleared, done set on request.
VXB_API int vxb_batcher_advance(vxb_batcher *b, int slot, int64_t n, int done) {
  if (!b) return set_error(nullptr, VXB_EINVAL, "vxb_batcher_advance: null batcher");
  if (slot < 0 || (size_t)slot >= b->slots.size() || !b->slots[slot].used)
    return set_error(nullptr, VXB_EINVAL, "vxb_batcher_advance: slot %d is empty", slot);
  auto &s = b->slots[slot];
  s.position += n;
  s.is_prefill = false;
  if (done) s.is_done = true;
  return VXB_OK;
}
