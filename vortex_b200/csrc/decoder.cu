// Llama-style decoder (stdlib/ai/transformer.vx:958-1156 semantics) built on
// the K1 GEMV, K4 decode attention and K5 kernels, one token per sequence per
// step, all weights Q4_0/Q8_0 in the tiled HBM layout, residual stream f32,
// KV cache paged (kv_cache.rs semantics). Each step is recorded once per batch
// size into a CUDA graph; host-side work per step is the KV block bookkeeping
// and one small upload of token ids and placements.
//
// Per layer (transformer_block, src ~ stdlib/ai/transformer.vx:958-1111):
//   h   = rmsnorm_bias(x)            -> bf16
//   qkv = [Wq;Wk;Wv] h               -> f32          (one fused GEMV)
//   q,k = rope(q,k, pos); v          -> bf16; k,v appended to the cache
//   a   = attention(q, cache)        -> bf16          (all cached tokens)
//   x  += Wo a                                        (GEMV epilogue adds x)
//   h   = rmsnorm_bias(x)            -> bf16
//   gu  = [W1;W3] h                  -> f32          (one fused GEMV)
//   x  += W2 bf16(silu(g) * u)                        (GEMV epilogue adds x)
// then logits = Wout rmsnorm_bias(x) and the greedy argmax (transformer.vx:
// 1120-1156, 1163-1177).
//
// Tensor parallel (vxb_decoder_create_tp, one process per GPU): rank r holds
// the q heads [r*H/tp, (r+1)*H/tp) and the matching kv heads (fused QKV rows
// and its KV cache), the gate/up rows [r*F/tp, (r+1)*F/tp), the matching
// input columns of Wo and W2, and the vocabulary rows [r*V/tp, (r+1)*V/tp) of
// the output projection. After the Wo and W2 GEMVs (rank 0 adds the residual
// in the epilogue) the residual stream is summed over ranks with an NCCL
// all-reduce, so every rank holds the full x for the norms; the greedy token
// is a max-reduction of (logit, index) keys. All collectives are recorded in
// the step's CUDA graph.
#include <algorithm>
#include <cmath>
#include <initializer_list>
#include <cstring>
#include <map>
#include <vector>

#include "comm.h"
#include "decode_attn.h"
#include "gemm.h"
#include "gemv.h"
#include "kv_cache.h"
#include "layer_ops.h"
#include "tiled_layout.h"

using namespace vxb;

struct vxb_decoder {
  vxb_ctx *ctx = nullptr;
  vxb_decoder_config cfg{};
  // this rank's slice: q / kv heads, q width, kv width (kvdim), ffn rows,
  // vocabulary rows; qkv_n = rows of the fused local QKV projection
  vxb_comm *comm = nullptr;
  int tp = 1, rank = 0;
  int hq = 0, hkv = 0, qdim = 0, kvdim = 0, ffn = 0, vocab = 0, qkv_n = 0;
  unsigned long long *d_keys = nullptr;           // [max_batch] argmax keys (tp > 1)
  float *logits_all = nullptr, *logits_full = nullptr;  // gathered shards (tp > 1)
  struct Layer {
    void *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr;
    float *ln1_w = nullptr, *ln1_b = nullptr, *ln2_w = nullptr, *ln2_b = nullptr;
  };
  std::vector<Layer> layers;
  uint16_t *emb = nullptr;
  float *lnf_w = nullptr, *lnf_b = nullptr;
  void *wlm = nullptr;
  double *rope_div = nullptr;
  vxb_kv *kv = nullptr;
  // activations sized for max_batch
  float *x = nullptr, *qkv = nullptr, *gu = nullptr, *logits = nullptr;
  uint16_t *h = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr;
  int32_t *d_tokens = nullptr, *d_next = nullptr, *d_slots = nullptr;
  KVPlace *d_places = nullptr;  // [n_layers][max_batch]
  float *attn_ws = nullptr;
  size_t attn_ws_bytes = 0;
  DecodePlan attn_plan[2]{};  // per distinct batch size captured (by key below)
  // Per-step uploads (placements [L][max_batch], slots [max_batch], tokens
  // [max_batch]) are staged in a ring of pinned buffers; a slot is reused only
  // after the event recorded behind its copy has completed, so the host can
  // plan step t+1 while step t is still queued.
  static constexpr int kRing = 4;
  struct Stage {
    uint8_t *host = nullptr;
    cudaEvent_t ev = nullptr;
    bool pending = false;
  };
  Stage ring[kRing];
  int ring_pos = 0;
  size_t stage_bytes = 0;
  uint8_t *d_stage = nullptr;
  int32_t *h_next = nullptr;
  KVPlace *h_places = nullptr;  // places of the stage being planned
  cudaStream_t stream = nullptr;
  struct Graph {
    cudaGraphExec_t exec = nullptr;
    std::vector<int64_t> seq_ids;
  };
  std::map<int, Graph> graphs;  // by batch size
  std::vector<void *> allocs;
  // prompt (prefill) activations, sized for the longest prompt seen
  struct Prefill {
    int cap = 0;
    float *x = nullptr, *qkv = nullptr, *gu = nullptr;
    uint16_t *h = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr, *act = nullptr;
    int32_t *tokens = nullptr;
    KVPlace *places = nullptr;     // [n_layers][cap]
    float *lse = nullptr;
    std::vector<void *> allocs;
  } pf;
};

namespace {

int dalloc(vxb_decoder *d, void **p, size_t bytes) {
  if (cudaMalloc(p, bytes) != cudaSuccess) {
    cudaGetLastError();
    *p = nullptr;
    return set_error(d->ctx, VXB_ENOMEM, "decoder: device allocation of %zu bytes failed", bytes);
  }
  d->allocs.push_back(*p);
  return VXB_OK;
}

template <typename T>
int dalloc_t(vxb_decoder *d, T **p, size_t count) {
  return dalloc(d, reinterpret_cast<void **>(p), count * sizeof(T));
}

__global__ void fill_f32_kernel(float *p, size_t n, float v) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

__global__ void f32_to_bf16_kernel(const float *in, size_t n, uint16_t *out) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = f32_to_bf16_bits(in[i]);
}

int fill(vxb_decoder *d, float *p, size_t n, float v) {
  fill_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, d->stream>>>(p, n, v);
  return launch_check(d->ctx, "fill_f32_kernel");
}

// One row block of a generated full matrix: rows [row0, row0 + rows) and
// columns [col0, col0 + cols) of the [*, ld] matrix of `seed`, placed at row
// `dst_row` of the local matrix.
struct GenPart {
  int dst_row, rows;
  size_t row0, col0, ld;
};

// Random N(0, sigma) weights of a local [N, K] matrix assembled from blocks of
// full matrices (the same values for every tensor-parallel layout), quantized
// to blocks and tiled.
int random_tiled(vxb_decoder *d, int N, int K, std::initializer_list<GenPart> parts, uint64_t seed, float sigma,
                 void **tiled) {
  const int fmt = d->cfg.weight_fmt;
  const size_t tb = vxb_tiled_bytes(fmt, N, K);
  if (int rc = dalloc(d, tiled, tb)) return rc;
  float *tmp = nullptr;
  uint8_t *blocks = nullptr;
  const size_t n = (size_t)N * K;
  if (cudaMalloc(&tmp, n * sizeof(float)) != cudaSuccess || cudaMalloc(&blocks, vxb_block_bytes(fmt, n)) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(tmp);
    cudaFree(blocks);
    return set_error(d->ctx, VXB_ENOMEM, "decoder: temporary allocation for weight generation failed");
  }
  int rc = VXB_OK;
  for (const GenPart &p : parts)
    if (!rc) rc = normal_fill_block(d->ctx, tmp + (size_t)p.dst_row * K, p.rows, K, p.row0, p.col0, p.ld, seed, sigma, d->stream);
  if (!rc) rc = vxb_quantize_blocks(d->ctx, fmt, tmp, n, blocks, d->stream);
  if (!rc) rc = vxb_tile_weights(d->ctx, fmt, blocks, N, K, *tiled, d->stream);
  cudaStreamSynchronize(d->stream);
  cudaFree(tmp);
  cudaFree(blocks);
  return rc;
}

int capture_step(vxb_decoder *d, int B, vxb_decoder::Graph &g);

}  // namespace

// ---------------------------------------------------------------- lifecycle

namespace {

int decoder_create(vxb_ctx *ctx, const vxb_decoder_config *cfg, vxb_comm *comm, vxb_decoder **out) {
  if (!ctx || !cfg || !out) return set_error(ctx, VXB_EINVAL, "vxb_decoder_create: null argument");
  *out = nullptr;
  const vxb_decoder_config &c = *cfg;
  if (c.vocab_size <= 0 || c.dim <= 0 || c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.ffn_dim <= 0 ||
      c.max_batch <= 0 || c.max_seq <= 0)
    return set_error(ctx, VXB_EINVAL, "vxb_decoder_create: sizes must be positive");
  if (c.dim % c.n_heads || c.n_heads % c.n_kv_heads)
    return set_error(ctx, VXB_EINVAL, "vxb_decoder_create: dim %% n_heads and n_heads %% n_kv_heads must be 0");
  const int hd = c.dim / c.n_heads;
  if (hd != 64 && hd != 128) return set_error(ctx, VXB_EUNSUPPORTED, "vxb_decoder_create: head_dim %d (64 or 128)", hd);
  if (c.dim % 32 || c.ffn_dim % 32) return set_error(ctx, VXB_EINVAL, "vxb_decoder_create: dim and ffn_dim must be multiples of 32");
  if (c.max_batch > 32) return set_error(ctx, VXB_EUNSUPPORTED, "vxb_decoder_create: max_batch %d > 32", c.max_batch);
  if (c.weight_fmt != VXB_Q4_0 && c.weight_fmt != VXB_Q8_0) return set_error(ctx, VXB_EINVAL, "vxb_decoder_create: weight_fmt");
  const int tp = comm ? comm->nranks : 1;
  if (c.n_heads % tp || c.n_kv_heads % tp || c.vocab_size % tp || (c.dim / tp) % 32 || (c.ffn_dim / tp) % 32 ||
      c.dim % tp || c.ffn_dim % tp)
    return set_error(ctx, VXB_EINVAL,
                     "vxb_decoder_create_tp: %d ranks must divide n_heads, n_kv_heads and vocab_size, and dim / ranks, "
                     "ffn_dim / ranks must be multiples of 32", tp);
  if (int rc = use_device(ctx)) return rc;
  vxb_decoder *d = new vxb_decoder();
  d->ctx = ctx;
  d->cfg = c;
  d->comm = comm;
  d->tp = tp;
  d->rank = comm ? comm->rank : 0;
  if (d->cfg.kv_block_size <= 0) d->cfg.kv_block_size = 16;
  if (d->cfg.norm_eps <= 0.f) d->cfg.norm_eps = 1e-5f;
  d->hq = c.n_heads / tp;
  d->hkv = c.n_kv_heads / tp;
  d->qdim = d->hq * hd;
  d->kvdim = d->hkv * hd;
  d->ffn = c.ffn_dim / tp;
  d->vocab = c.vocab_size / tp;
  d->qkv_n = d->qdim + 2 * d->kvdim;
  int rc = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking) == cudaSuccess ? VXB_OK : VXB_ECUDA;
  const int B = c.max_batch, L = c.n_layers;
  if (!rc) rc = dalloc_t(d, &d->x, (size_t)B * c.dim);
  if (!rc) rc = dalloc_t(d, &d->qkv, (size_t)B * d->qkv_n);
  if (!rc) rc = dalloc_t(d, &d->gu, (size_t)B * 2 * d->ffn);
  if (!rc) rc = dalloc_t(d, &d->logits, (size_t)B * d->vocab);
  if (!rc) rc = dalloc_t(d, &d->h, (size_t)B * (c.dim > c.ffn_dim ? c.dim : c.ffn_dim));
  if (!rc) rc = dalloc_t(d, &d->q, (size_t)B * d->qdim);
  if (!rc) rc = dalloc_t(d, &d->attn, (size_t)B * d->qdim);
  if (!rc) rc = dalloc_t(d, &d->act, (size_t)B * d->ffn);
  if (!rc && tp > 1) rc = dalloc_t(d, &d->d_keys, (size_t)B);
  if (!rc && tp > 1) rc = dalloc_t(d, &d->logits_all, (size_t)B * c.vocab_size);
  if (!rc && tp > 1) rc = dalloc_t(d, &d->logits_full, (size_t)B * c.vocab_size);
  d->stage_bytes = (size_t)L * B * sizeof(KVPlace) + 2 * (size_t)B * sizeof(int32_t);
  if (!rc) rc = dalloc(d, (void **)&d->d_stage, d->stage_bytes);
  if (!rc) {
    d->d_places = (KVPlace *)d->d_stage;
    d->d_slots = (int32_t *)(d->d_stage + (size_t)L * B * sizeof(KVPlace));
    d->d_tokens = d->d_slots + B;
  }
  if (!rc) rc = dalloc_t(d, &d->d_next, (size_t)B);
  if (!rc) rc = dalloc_t(d, &d->rope_div, (size_t)(c.dim / 2 > d->kvdim / 2 ? c.dim / 2 : d->kvdim / 2));
  if (!rc) {
    // divisor exp(i * ln(10000) / dim) per pair (transformer.vx:442-466), on the host in f64
    std::vector<double> div((size_t)c.dim / 2);
    for (int i = 0; i < c.dim / 2; i++) div[i] = std::exp((double)i * std::log(10000.0) / (double)c.dim);
    rc = cudaMemcpy(d->rope_div, div.data(), div.size() * sizeof(double), cudaMemcpyHostToDevice) == cudaSuccess
             ? VXB_OK : set_error(ctx, VXB_ECUDA, "decoder: rope table upload failed");
  }
  if (!rc && cudaMallocHost(&d->h_next, B * sizeof(int32_t)) != cudaSuccess)
    rc = set_error(ctx, VXB_ENOMEM, "decoder: pinned host allocation failed");
  for (int i = 0; i < vxb_decoder::kRing && !rc; i++) {
    if (cudaMallocHost(&d->ring[i].host, d->stage_bytes) != cudaSuccess ||
        cudaEventCreateWithFlags(&d->ring[i].ev, cudaEventDisableTiming) != cudaSuccess)
      rc = set_error(ctx, VXB_ENOMEM, "decoder: pinned staging allocation failed");
  }
  if (!rc) {
    const int bs = d->cfg.kv_block_size;
    const int mbps = (c.max_seq + bs - 1) / bs;
    const int max_blocks = L * B * mbps;
    rc = vxb_kv_create(ctx, L, d->hkv, hd, bs, max_blocks, B, mbps, c.kv_dtype ? c.kv_dtype : VXB_BF16, &d->kv);
  }
  if (!rc) {
    // attention scratch for the largest batch at the largest split count any
    // plan uses, so that every captured step fits
    d->attn_ws_bytes = decode_ws_bytes(B, d->hkv, c.n_heads / c.n_kv_heads, hd, kMaxDecodeSplits);
    rc = dalloc(d, (void **)&d->attn_ws, d->attn_ws_bytes);
  }
  if (!rc) {
    // GEMV split-K partials for the widest projection (at most 16 splits), so
    // that recording a step into a graph never allocates
    size_t widest = (size_t)std::max(std::max(std::max(2 * d->ffn, d->vocab), d->qkv_n), c.dim) + 16;
    rc = ws_reserve(ctx, (size_t)32 * B * widest * 4, (size_t)B * c.n_kv_heads + 65536);
  }
  d->layers.resize(L);
  if (rc) {
    vxb_decoder_destroy(d);
    return rc;
  }
  *out = d;
  return VXB_OK;
}

}  // namespace

VXB_API int vxb_decoder_create(vxb_ctx *ctx, const vxb_decoder_config *cfg, vxb_decoder **out) {
  return decoder_create(ctx, cfg, nullptr, out);
}

VXB_API int vxb_decoder_create_tp(vxb_ctx *ctx, const vxb_decoder_config *cfg, vxb_comm *comm, vxb_decoder **out) {
  if (!comm) return set_error(ctx, VXB_EINVAL, "vxb_decoder_create_tp: null communicator");
  if (comm->ctx != ctx) return set_error(ctx, VXB_EINVAL, "vxb_decoder_create_tp: communicator of another context");
  return decoder_create(ctx, cfg, comm, out);
}

VXB_API int vxb_decoder_destroy(vxb_decoder *d) {
  if (!d) return VXB_OK;
  if (d->ctx) use_device(d->ctx);
  for (auto &kvp : d->graphs)
    if (kvp.second.exec) cudaGraphExecDestroy(kvp.second.exec);
  if (d->kv) vxb_kv_destroy(d->kv);
  for (void *p : d->allocs) cudaFree(p);
  for (void *p : d->pf.allocs) cudaFree(p);
  if (d->h_next) cudaFreeHost(d->h_next);
  for (auto &s : d->ring) {
    if (s.host) cudaFreeHost(s.host);
    if (s.ev) cudaEventDestroy(s.ev);
  }
  if (d->stream) cudaStreamDestroy(d->stream);
  delete d;
  return VXB_OK;
}

// Synthetic weights: every linear N(0, sigma) quantized to the weight format,
// norms w = 1, b = 0, embedding N(0, sigma) in bf16 (init_random_weights,
// stdlib/ai/transformer.vx:661-725, with a counter-based generator).
VXB_API int vxb_decoder_init_random(vxb_decoder *d, uint64_t seed, float sigma) {
  if (!d) return set_error(nullptr, VXB_EINVAL, "vxb_decoder_init_random: null decoder");
  if (int rc = use_device(d->ctx)) return rc;
  const vxb_decoder_config &c = d->cfg;
  uint64_t s = seed;
  const int r = d->rank, kvfull = c.n_kv_heads * (c.dim / c.n_heads);
  const size_t D = c.dim, F = c.ffn_dim;
  for (int l = 0; l < c.n_layers; l++) {
    auto &L = d->layers[l];
    // full fused QKV [dim + 2 kvdim, dim]: this rank's q, k and v rows
    int rc = random_tiled(d, d->qkv_n, c.dim,
                          {{0, d->qdim, (size_t)r * d->qdim, 0, D},
                           {d->qdim, d->kvdim, D + (size_t)r * d->kvdim, 0, D},
                           {d->qdim + d->kvdim, d->kvdim, D + kvfull + (size_t)r * d->kvdim, 0, D}},
                          ++s, sigma, &L.wqkv);
    // full Wo [dim, dim]: this rank's input columns
    if (!rc) rc = random_tiled(d, c.dim, d->qdim, {{0, c.dim, 0, (size_t)r * d->qdim, D}}, ++s, sigma, &L.wo);
    // full [W1; W3] [2 ffn, dim]: this rank's gate and up rows
    if (!rc)
      rc = random_tiled(d, 2 * d->ffn, c.dim, {{0, d->ffn, (size_t)r * d->ffn, 0, D}, {d->ffn, d->ffn, F + (size_t)r * d->ffn, 0, D}},
                        ++s, sigma, &L.wgu);
    // full W2 [dim, ffn]: this rank's input columns
    if (!rc) rc = random_tiled(d, c.dim, d->ffn, {{0, c.dim, 0, (size_t)r * d->ffn, F}}, ++s, sigma, &L.wdown);
    for (float **p : {&L.ln1_w, &L.ln1_b, &L.ln2_w, &L.ln2_b})
      if (!rc) rc = dalloc_t(d, p, (size_t)c.dim);
    if (!rc) rc = fill(d, L.ln1_w, c.dim, 1.f);
    if (!rc) rc = fill(d, L.ln1_b, c.dim, 0.f);
    if (!rc) rc = fill(d, L.ln2_w, c.dim, 1.f);
    if (!rc) rc = fill(d, L.ln2_b, c.dim, 0.f);
    if (rc) return rc;
  }
  int rc = dalloc_t(d, &d->emb, (size_t)c.vocab_size * c.dim);
  if (!rc) {
    float *tmp = nullptr;
    const size_t n = (size_t)c.vocab_size * c.dim;
    if (cudaMalloc(&tmp, n * 4) != cudaSuccess) {
      cudaGetLastError();
      return set_error(d->ctx, VXB_ENOMEM, "decoder: embedding temporary");
    }
    rc = normal_fill(d->ctx, tmp, n, ++s, 0, sigma, d->stream);
    f32_to_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, d->stream>>>(tmp, n, d->emb);
    cudaStreamSynchronize(d->stream);
    cudaFree(tmp);
  }
  if (!rc) rc = dalloc_t(d, &d->lnf_w, (size_t)c.dim);
  if (!rc) rc = dalloc_t(d, &d->lnf_b, (size_t)c.dim);
  if (!rc) rc = fill(d, d->lnf_w, c.dim, 1.f);
  if (!rc) rc = fill(d, d->lnf_b, c.dim, 0.f);
  if (!rc) rc = random_tiled(d, d->vocab, c.dim, {{0, d->vocab, (size_t)r * d->vocab, 0, D}}, ++s, sigma, &d->wlm);
  if (!rc) VXB_CUDA_TRY(d->ctx, cudaStreamSynchronize(d->stream));
  return rc;
}

// Weights from host buffers: which = 0 wq, 1 wk, 2 wv, 3 wo, 4 w1, 5 w2, 6 w3
// (GGUF blocks, row-major [out, in]); 7..10 ln1_w, ln1_b, ln2_w, ln2_b (f32);
// layer -1: 0 embedding (bf16 bits [vocab, dim]), 1 final_w, 2 final_b (f32),
// 3 output projection (blocks [vocab, dim]). wq/wk/wv and w1/w3 are fused on
// the device; load all three (two) before the first step.
VXB_API int vxb_decoder_set_weight(vxb_decoder *d, int layer, int which, const void *h_data, size_t bytes) {
  if (!d || !h_data) return set_error(d ? d->ctx : nullptr, VXB_EINVAL, "vxb_decoder_set_weight: null argument");
  if (int rc = use_device(d->ctx)) return rc;
  const vxb_decoder_config &c = d->cfg;
  const int fmt = c.weight_fmt;
  // Upload rows [row0, row0 + nrows) of a local [N_total, K] matrix from
  // GGUF blocks; `src` holds those rows, `src_bytes` their size.
  auto upload_blocks = [&](void **tiled, int N_total, int K, int row0, int nrows, const void *src,
                           size_t src_bytes) -> int {
    if (!*tiled) {
      if (int rc = dalloc(d, tiled, vxb_tiled_bytes(fmt, N_total, K))) return rc;
      if (int rc = tile_header(d->ctx, fmt, N_total, K, *tiled, d->stream)) return rc;
    }
    uint8_t *blocks = nullptr;
    if (cudaMalloc(&blocks, src_bytes) != cudaSuccess) {
      cudaGetLastError();
      return set_error(d->ctx, VXB_ENOMEM, "vxb_decoder_set_weight: staging");
    }
    VXB_CUDA_TRY(d->ctx, cudaMemcpyAsync(blocks, src, src_bytes, cudaMemcpyHostToDevice, d->stream));
    int rc = tile_part(d->ctx, fmt, blocks, nrows, K, row0, N_total, *tiled, d->stream);
    cudaStreamSynchronize(d->stream);
    cudaFree(blocks);
    return rc;
  };
  // A full [rows_full, K_full] host matrix (GGUF blocks) of which this rank
  // keeps rows [r0, r0 + nr) and columns [k0, k0 + nk) (multiples of 32).
  std::vector<uint8_t> slice;
  auto upload_tiled_part = [&](void **tiled, int N_total, int row0, int rows_full, int K_full, int r0, int nr, int k0,
                               int nk) -> int {
    const size_t bpr = vxb_block_bytes(fmt, (size_t)K_full);  // bytes per full row
    if (bytes != bpr * rows_full)
      return set_error(d->ctx, VXB_EINVAL, "vxb_decoder_set_weight: expected %zu bytes, got %zu", bpr * rows_full, bytes);
    const uint8_t *src = (const uint8_t *)h_data + (size_t)r0 * bpr;
    if (nk == K_full) return upload_blocks(tiled, N_total, nk, row0, nr, src, bpr * nr);
    const size_t bb = vxb_block_bytes(fmt, 32), off = (size_t)(k0 / 32) * bb, len = (size_t)(nk / 32) * bb;
    slice.resize(len * nr);
    for (int i = 0; i < nr; i++) std::memcpy(slice.data() + (size_t)i * len, src + (size_t)i * bpr + off, len);
    return upload_blocks(tiled, N_total, nk, row0, nr, slice.data(), slice.size());
  };
  auto upload_f32 = [&](float **p, size_t n) -> int {
    if (bytes != n * 4) return set_error(d->ctx, VXB_EINVAL, "vxb_decoder_set_weight: expected %zu bytes", n * 4);
    if (!*p)
      if (int rc = dalloc_t(d, p, n)) return rc;
    VXB_CUDA_TRY(d->ctx, cudaMemcpy(*p, h_data, bytes, cudaMemcpyHostToDevice));
    return VXB_OK;
  };
  if (layer == -1) {
    switch (which) {
      case 0: {
        const size_t n = (size_t)c.vocab_size * c.dim;
        if (bytes != n * 2) return set_error(d->ctx, VXB_EINVAL, "vxb_decoder_set_weight: embedding size");
        if (!d->emb)
          if (int rc = dalloc_t(d, &d->emb, n)) return rc;
        VXB_CUDA_TRY(d->ctx, cudaMemcpy(d->emb, h_data, bytes, cudaMemcpyHostToDevice));
        return VXB_OK;
      }
      case 1: return upload_f32(&d->lnf_w, c.dim);
      case 2: return upload_f32(&d->lnf_b, c.dim);
      case 3:
        return upload_tiled_part(&d->wlm, d->vocab, 0, c.vocab_size, c.dim, d->rank * d->vocab, d->vocab, 0, c.dim);
      default: return set_error(d->ctx, VXB_EINVAL, "vxb_decoder_set_weight: which %d", which);
    }
  }
  if (layer < 0 || layer >= c.n_layers) return set_error(d->ctx, VXB_EINVAL, "vxb_decoder_set_weight: layer %d", layer);
  auto &L = d->layers[layer];
  const int r = d->rank, kvfull = c.n_kv_heads * (c.dim / c.n_heads);
  switch (which) {
    // column-parallel (this rank's output rows) and row-parallel (this rank's
    // input columns) slices of the full matrices
    case 0: return upload_tiled_part(&L.wqkv, d->qkv_n, 0, c.dim, c.dim, r * d->qdim, d->qdim, 0, c.dim);
    case 1: return upload_tiled_part(&L.wqkv, d->qkv_n, d->qdim, kvfull, c.dim, r * d->kvdim, d->kvdim, 0, c.dim);
    case 2:
      return upload_tiled_part(&L.wqkv, d->qkv_n, d->qdim + d->kvdim, kvfull, c.dim, r * d->kvdim, d->kvdim, 0, c.dim);
    case 3: return upload_tiled_part(&L.wo, c.dim, 0, c.dim, c.dim, 0, c.dim, r * d->qdim, d->qdim);
    case 4: return upload_tiled_part(&L.wgu, 2 * d->ffn, 0, c.ffn_dim, c.dim, r * d->ffn, d->ffn, 0, c.dim);
    case 5: return upload_tiled_part(&L.wdown, c.dim, 0, c.dim, c.ffn_dim, 0, c.dim, r * d->ffn, d->ffn);
    case 6: return upload_tiled_part(&L.wgu, 2 * d->ffn, d->ffn, c.ffn_dim, c.dim, r * d->ffn, d->ffn, 0, c.dim);
    case 7: return upload_f32(&L.ln1_w, c.dim);
    case 8: return upload_f32(&L.ln1_b, c.dim);
    case 9: return upload_f32(&L.ln2_w, c.dim);
    case 10: return upload_f32(&L.ln2_b, c.dim);
    default: return set_error(d->ctx, VXB_EINVAL, "vxb_decoder_set_weight: which %d", which);
  }
}

namespace {

// Record the device part of one step for batch B on d->stream.
int record_step(vxb_decoder *d, int B) {
  const vxb_decoder_config &c = d->cfg;
  vxb_ctx *ctx = d->ctx;
  cudaStream_t st = d->stream;
  const int hd = c.dim / c.n_heads;
  const float eps = d->cfg.norm_eps;
  const float scale = 1.0f / sqrtf((float)hd);
  const int fmt = c.weight_fmt;
  const DecodePlan ap = decode_plan(ctx, B, d->hkv, c.max_seq);
  if (decode_ws_bytes(B, d->hkv, c.n_heads / c.n_kv_heads, hd, ap.splits) > d->attn_ws_bytes)
    return set_error(ctx, VXB_EINVAL, "decoder: attention scratch too small");
  int rc = embed_launch(ctx, d->emb, d->d_tokens, B, c.dim, c.vocab_size, d->x, st);
  for (int l = 0; l < c.n_layers && !rc; l++) {
    auto &L = d->layers[l];
    rc = rmsnorm_launch(ctx, d->x, L.ln1_w, L.ln1_b, B, c.dim, eps, d->h, st);
    if (!rc) rc = gemv_launch(ctx, fmt, L.wqkv, d->qkv_n, c.dim, d->h, B, VXB_F32, d->qkv, nullptr, st, nullptr);
    if (!rc)
      rc = rope_kv_launch(ctx, d->kv, l, d->qkv, B, d->qdim, d->kvdim, hd, d->d_places + (size_t)l * c.max_batch,
                          d->rope_div, d->q, nullptr, nullptr, d->rank * d->qdim / 2, d->rank * d->kvdim / 2, st);
    if (!rc)
      rc = decode_attn_launch(d->kv, l, B, d->d_slots, nullptr, d->q, d->hq, scale, d->attn, nullptr, ap, d->attn_ws, st);
    // row-parallel Wo: rank 0 adds the residual, the partials are summed over ranks
    if (!rc) rc = gemv_launch(ctx, fmt, L.wo, c.dim, d->qdim, d->attn, B, VXB_F32, d->x, d->rank == 0 ? d->x : nullptr, st, nullptr);
    if (!rc && d->tp > 1) rc = comm_allreduce(d->comm, d->x, (size_t)B * c.dim, VXB_F32, 0, st);
    if (!rc) rc = rmsnorm_launch(ctx, d->x, L.ln2_w, L.ln2_b, B, c.dim, eps, d->h, st);
    if (!rc) rc = gemv_launch(ctx, fmt, L.wgu, 2 * d->ffn, c.dim, d->h, B, VXB_F32, d->gu, nullptr, st, nullptr);
    if (!rc) rc = swiglu_launch(ctx, d->gu, B, d->ffn, d->act, st);
    if (!rc) rc = gemv_launch(ctx, fmt, L.wdown, c.dim, d->ffn, d->act, B, VXB_F32, d->x, d->rank == 0 ? d->x : nullptr, st, nullptr);
    if (!rc && d->tp > 1) rc = comm_allreduce(d->comm, d->x, (size_t)B * c.dim, VXB_F32, 0, st);
  }
  if (!rc) rc = rmsnorm_launch(ctx, d->x, d->lnf_w, d->lnf_b, B, c.dim, eps, d->h, st);
  if (!rc) rc = gemv_launch(ctx, fmt, d->wlm, d->vocab, c.dim, d->h, B, VXB_F32, d->logits, nullptr, st, nullptr);
  if (d->tp == 1) {
    if (!rc) rc = argmax_launch(ctx, d->logits, B, c.vocab_size, d->d_next, st);
  } else {
    // first maximum over the vocabulary shards: max-reduce (logit, index) keys
    if (!rc) rc = argmax_key_launch(ctx, d->logits, B, d->vocab, d->rank * d->vocab, d->d_keys, st);
    if (!rc) rc = comm_allreduce(d->comm, d->d_keys, (size_t)B, -1, 1, st);
    if (!rc) rc = key_to_token_launch(ctx, d->d_keys, B, d->d_next, st);
  }
  return rc;
}

int capture_step(vxb_decoder *d, int B, vxb_decoder::Graph &g) {
  cudaGraph_t graph = nullptr;
  VXB_CUDA_TRY(d->ctx, cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal));
  int rc = record_step(d, B);
  cudaError_t e = cudaStreamEndCapture(d->stream, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return cuda_fail(d->ctx, e, "cudaStreamEndCapture");
  e = cudaGraphInstantiate(&g.exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return cuda_fail(d->ctx, e, "cudaGraphInstantiate");
  return VXB_OK;
}

// Host bookkeeping of one step: slots and placements for every layer.
int plan_step(vxb_decoder *d, int B, const int64_t *seq_ids) {
  const vxb_decoder_config &c = d->cfg;
  for (int l = 0; l < c.n_layers; l++) {
    for (int b = 0; b < B; b++) {
      if (int rc = kv_place(d->kv, l, seq_ids[b], &d->h_places[(size_t)l * c.max_batch + b])) {
        // roll back this step's placements
        for (int bb = b - 1; bb >= 0; bb--) kv_unplace(d->kv, l, seq_ids[bb], 1);
        for (int ll = l - 1; ll >= 0; ll--)
          for (int bb = B - 1; bb >= 0; bb--) kv_unplace(d->kv, ll, seq_ids[bb], 1);
        return rc;
      }
    }
  }
  // every layer of a sequence uses the same slot and position
  for (int b = 0; b < B; b++) {
    const int32_t pos0 = d->h_places[b].pos;
    for (int l = 1; l < c.n_layers; l++)
      if (d->h_places[(size_t)l * c.max_batch + b].pos != pos0)
        return set_error(d->ctx, VXB_EINVAL, "decoder: sequence %lld has layers of different lengths",
                         (long long)seq_ids[b]);
  }
  return VXB_OK;
}

int launch_step(vxb_decoder *d, int B, const int64_t *seq_ids, const int32_t *d_tokens_in, bool tokens_on_host,
                const int32_t *h_tokens_in) {
  const vxb_decoder_config &c = d->cfg;
  if (B <= 0 || B > c.max_batch) return set_error(d->ctx, VXB_EINVAL, "decoder: batch %d outside 1..%d", B, c.max_batch);
  if (!d->emb || !d->wlm || !d->layers[0].wqkv) return set_error(d->ctx, VXB_EINVAL, "decoder: weights not loaded");
  for (int i = 0; i < B; i++)
    for (int j = 0; j < i; j++)
      if (seq_ids[i] == seq_ids[j]) return set_error(d->ctx, VXB_EINVAL, "decoder: sequence listed twice");
  if (int rc = use_device(d->ctx)) return rc;
  auto it = d->graphs.find(B);
  if (it == d->graphs.end()) {
    vxb_decoder::Graph g;
    if (int rc = capture_step(d, B, g)) return rc;
    it = d->graphs.emplace(B, g).first;
  }
  vxb_decoder::Stage &s = d->ring[d->ring_pos];
  if (s.pending) VXB_CUDA_TRY(d->ctx, cudaEventSynchronize(s.ev));
  s.pending = false;
  d->h_places = (KVPlace *)s.host;
  if (int rc = plan_step(d, B, seq_ids)) return rc;
  d->ring_pos = (d->ring_pos + 1) % vxb_decoder::kRing;
  // placements, slots (fixed per sequence) and host tokens in one copy
  const size_t pl_bytes = (size_t)c.n_layers * c.max_batch * sizeof(KVPlace);
  int32_t *slots = (int32_t *)(s.host + pl_bytes);
  for (int b = 0; b < B; b++) slots[b] = d->h_places[b].slot;
  size_t bytes = pl_bytes + (size_t)c.max_batch * sizeof(int32_t);
  if (tokens_on_host) {
    std::memcpy(slots + c.max_batch, h_tokens_in, B * sizeof(int32_t));
    bytes += B * sizeof(int32_t);
  }
  cudaStream_t st = d->stream;
  VXB_CUDA_TRY(d->ctx, cudaMemcpyAsync(d->d_stage, s.host, bytes, cudaMemcpyHostToDevice, st));
  VXB_CUDA_TRY(d->ctx, cudaEventRecord(s.ev, st));
  s.pending = true;
  if (!tokens_on_host && d_tokens_in != d->d_tokens)
    VXB_CUDA_TRY(d->ctx, cudaMemcpyAsync(d->d_tokens, d_tokens_in, B * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  VXB_CUDA_TRY(d->ctx, cudaGraphLaunch(it->second.exec, st));
  return VXB_OK;
}

}  // namespace

namespace {

int pf_alloc(vxb_decoder *d, void **p, size_t bytes) {
  if (cudaMalloc(p, bytes) != cudaSuccess) {
    cudaGetLastError();
    *p = nullptr;
    return set_error(d->ctx, VXB_ENOMEM, "decoder prefill: device allocation of %zu bytes failed", bytes);
  }
  d->pf.allocs.push_back(*p);
  return VXB_OK;
}

template <typename T>
int pf_alloc_t(vxb_decoder *d, T **p, size_t count) {
  return pf_alloc(d, reinterpret_cast<void **>(p), count * sizeof(T));
}

int pf_reserve(vxb_decoder *d, int n) {
  auto &P = d->pf;
  if (n <= P.cap) return VXB_OK;
  VXB_CUDA_TRY(d->ctx, cudaStreamSynchronize(d->stream));
  for (void *p : P.allocs) cudaFree(p);
  P.allocs.clear();
  P.cap = 0;
  const vxb_decoder_config &c = d->cfg;
  const size_t N = (size_t)n;
  int rc = pf_alloc_t(d, &P.x, N * c.dim);
  if (!rc) rc = pf_alloc_t(d, &P.qkv, N * d->qkv_n);
  if (!rc) rc = pf_alloc_t(d, &P.gu, N * 2 * d->ffn);
  if (!rc) rc = pf_alloc_t(d, &P.h, N * c.dim);
  if (!rc) rc = pf_alloc_t(d, &P.q, N * d->qdim);
  if (!rc) rc = pf_alloc_t(d, &P.k, N * d->kvdim);
  if (!rc) rc = pf_alloc_t(d, &P.v, N * d->kvdim);
  if (!rc) rc = pf_alloc_t(d, &P.attn, N * d->qdim);
  if (!rc) rc = pf_alloc_t(d, &P.act, N * d->ffn);
  if (!rc) rc = pf_alloc_t(d, &P.tokens, N);
  if (!rc) rc = pf_alloc_t(d, &P.places, N * c.n_layers);
  if (!rc) rc = pf_alloc_t(d, &P.lse, N * d->hq);
  if (!rc) P.cap = n;
  return rc;
}

}  // namespace

// Prompt of n tokens for a new sequence in one pass (prefill): every
// projection is a K2 GEMM over the n rows, attention is the causal K3 flash
// kernel over the prompt, and the K/V of all n positions enter the cache.
// h_next (optional) gets the greedy next token, h_logits (optional) the
// logits [vocab] of the last position. Synchronous. With tensor parallelism
// every rank calls it with the same arguments.
VXB_API int vxb_decoder_prefill(vxb_decoder *d, int64_t seq_id, const int32_t *h_tokens, int n, int32_t *h_next,
                                float *h_logits) {
  if (!d || !h_tokens) return set_error(d ? d->ctx : nullptr, VXB_EINVAL, "vxb_decoder_prefill: null argument");
  const vxb_decoder_config &c = d->cfg;
  vxb_ctx *ctx = d->ctx;
  if (n < 1 || n > c.max_seq) return set_error(ctx, VXB_EINVAL, "vxb_decoder_prefill: %d tokens (1..%d)", n, c.max_seq);
  if (c.dim / c.n_heads != 128)
    return set_error(ctx, VXB_EUNSUPPORTED, "vxb_decoder_prefill: head_dim %d (the prefill attention needs 128)",
                     c.dim / c.n_heads);
  if (!d->emb || !d->wlm || !d->layers[0].wqkv) return set_error(ctx, VXB_EINVAL, "decoder: weights not loaded");
  for (int i = 0; i < n; i++)
    if (h_tokens[i] < 0 || h_tokens[i] >= c.vocab_size)
      return set_error(ctx, VXB_EINVAL, "vxb_decoder_prefill: token %d out of range", h_tokens[i]);
  if (int rc = use_device(ctx)) return rc;
  for (int l = 0; l < c.n_layers; l++) {
    auto it = d->kv->tables.find(std::make_pair(l, seq_id));
    if (it != d->kv->tables.end() && it->second.len > 0)
      return set_error(ctx, VXB_EINVAL, "vxb_decoder_prefill: sequence %lld already holds tokens", (long long)seq_id);
  }
  cudaStream_t st = d->stream;
  // any queued decode step still reads the staging ring and activations
  VXB_CUDA_TRY(ctx, cudaStreamSynchronize(st));
  if (int rc = pf_reserve(d, n)) return rc;
  auto &P = d->pf;
  // KV placements of every position in every layer (host allocator)
  std::vector<KVPlace> pl((size_t)n * c.n_layers);
  for (int l = 0; l < c.n_layers; l++)
    for (int i = 0; i < n; i++)
      if (int rc = kv_place(d->kv, l, seq_id, &pl[(size_t)l * n + i])) {
        kv_unplace(d->kv, l, seq_id, i);
        for (int ll = l - 1; ll >= 0; ll--) kv_unplace(d->kv, ll, seq_id, n);
        return rc;
      }
  VXB_CUDA_TRY(ctx, cudaMemcpyAsync(P.places, pl.data(), pl.size() * sizeof(KVPlace), cudaMemcpyHostToDevice, st));
  VXB_CUDA_TRY(ctx, cudaMemcpyAsync(P.tokens, h_tokens, (size_t)n * sizeof(int32_t), cudaMemcpyHostToDevice, st));
  size_t scratch_bytes = std::max(std::max(gemm_scratch_bytes(d->qkv_n, c.dim), gemm_scratch_bytes(c.dim, d->qdim)),
                                  std::max(gemm_scratch_bytes(2 * d->ffn, c.dim), gemm_scratch_bytes(c.dim, d->ffn)));
  void *scratch = nullptr;
  if (int rc = gemm_ws_reserve(ctx, scratch_bytes, &scratch)) return rc;
  const int fmt = c.weight_fmt;
  const float eps = c.norm_eps, scale = 1.0f / sqrtf(128.f);
  int rc = embed_launch(ctx, d->emb, P.tokens, n, c.dim, c.vocab_size, P.x, st);
  for (int l = 0; l < c.n_layers && !rc; l++) {
    auto &L = d->layers[l];
    rc = rmsnorm_launch(ctx, P.x, L.ln1_w, L.ln1_b, n, c.dim, eps, P.h, st);
    if (!rc) rc = gemm_q_launch(ctx, fmt, L.wqkv, d->qkv_n, c.dim, P.h, n, VXB_F32, P.qkv, nullptr, scratch, st);
    if (!rc)
      rc = rope_kv_launch(ctx, d->kv, l, P.qkv, n, d->qdim, d->kvdim, 128, P.places + (size_t)l * n, d->rope_div, P.q,
                          P.k, P.v, d->rank * d->qdim / 2, d->rank * d->kvdim / 2, st);
    if (!rc)
      rc = vxb_flash_fwd(ctx, P.q, P.k, P.v, 1, d->hq, d->hkv, n, 128, scale, 1, P.attn, P.lse, st);
    if (!rc)
      rc = gemm_q_launch(ctx, fmt, L.wo, c.dim, d->qdim, P.attn, n, VXB_F32, P.x, d->rank == 0 ? P.x : nullptr, scratch, st);
    if (!rc && d->tp > 1) rc = comm_allreduce(d->comm, P.x, (size_t)n * c.dim, VXB_F32, 0, st);
    if (!rc) rc = rmsnorm_launch(ctx, P.x, L.ln2_w, L.ln2_b, n, c.dim, eps, P.h, st);
    if (!rc) rc = gemm_q_launch(ctx, fmt, L.wgu, 2 * d->ffn, c.dim, P.h, n, VXB_F32, P.gu, nullptr, scratch, st);
    if (!rc) rc = swiglu_launch(ctx, P.gu, n, d->ffn, P.act, st);
    if (!rc)
      rc = gemm_q_launch(ctx, fmt, L.wdown, c.dim, d->ffn, P.act, n, VXB_F32, P.x, d->rank == 0 ? P.x : nullptr, scratch, st);
    if (!rc && d->tp > 1) rc = comm_allreduce(d->comm, P.x, (size_t)n * c.dim, VXB_F32, 0, st);
  }
  // the last position's logits and greedy token (decode-step buffers, row 0)
  const float *xl = P.x + (size_t)(n - 1) * c.dim;
  if (!rc) rc = rmsnorm_launch(ctx, xl, d->lnf_w, d->lnf_b, 1, c.dim, eps, d->h, st);
  if (!rc) rc = gemv_launch(ctx, fmt, d->wlm, d->vocab, c.dim, d->h, 1, VXB_F32, d->logits, nullptr, st, nullptr);
  if (d->tp == 1) {
    if (!rc) rc = argmax_launch(ctx, d->logits, 1, c.vocab_size, d->d_next, st);
  } else {
    if (!rc) rc = argmax_key_launch(ctx, d->logits, 1, d->vocab, d->rank * d->vocab, d->d_keys, st);
    if (!rc) rc = comm_allreduce(d->comm, d->d_keys, 1, -1, 1, st);
    if (!rc) rc = key_to_token_launch(ctx, d->d_keys, 1, d->d_next, st);
  }
  if (rc) return rc;
  if (h_logits) {
    const float *src = d->logits;
    if (d->tp > 1) {
      if (int r2 = comm_allgather_f32(d->comm, d->logits, d->logits_all, (size_t)d->vocab, st)) return r2;
      if (int r2 = unshard_launch(ctx, d->logits_all, d->tp, 1, d->vocab, d->logits_full, st)) return r2;
      src = d->logits_full;
    }
    VXB_CUDA_TRY(ctx, cudaMemcpyAsync(h_logits, src, (size_t)c.vocab_size * sizeof(float), cudaMemcpyDeviceToHost, st));
  }
  if (h_next) VXB_CUDA_TRY(ctx, cudaMemcpyAsync(d->h_next, d->d_next, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  VXB_CUDA_TRY(ctx, cudaStreamSynchronize(st));
  if (h_next) *h_next = d->h_next[0];
  return VXB_OK;
}

// One decode step through host buffers: h_tokens [B] in, h_next [B] out
// (greedy argmax), optional h_logits [B, vocab]. Synchronous.
VXB_API int vxb_decoder_step(vxb_decoder *d, int batch, const int64_t *h_seq_ids, const int32_t *h_tokens,
                             int32_t *h_next, float *h_logits) {
  if (!d || !h_seq_ids || !h_tokens || !h_next) return set_error(d ? d->ctx : nullptr, VXB_EINVAL, "vxb_decoder_step: null argument");
  if (int rc = launch_step(d, batch, h_seq_ids, nullptr, true, h_tokens)) return rc;
  cudaStream_t st = d->stream;
  VXB_CUDA_TRY(d->ctx, cudaMemcpyAsync(d->h_next, d->d_next, batch * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  if (h_logits) {
    const float *src = d->logits;
    if (d->tp > 1) {
      if (int rc = comm_allgather_f32(d->comm, d->logits, d->logits_all, (size_t)batch * d->vocab, st)) return rc;
      if (int rc = unshard_launch(d->ctx, d->logits_all, d->tp, batch, d->vocab, d->logits_full, st)) return rc;
      src = d->logits_full;
    }
    VXB_CUDA_TRY(d->ctx, cudaMemcpyAsync(h_logits, src, (size_t)batch * d->cfg.vocab_size * sizeof(float),
                                         cudaMemcpyDeviceToHost, st));
  }
  VXB_CUDA_TRY(d->ctx, cudaStreamSynchronize(st));
  std::memcpy(h_next, d->h_next, batch * sizeof(int32_t));
  return VXB_OK;
}

// One decode step with device buffers, asynchronous on the decoder's stream
// (which is ordered after `stream` on entry and before it on return).
VXB_API int vxb_decoder_step_device(vxb_decoder *d, int batch, const int64_t *h_seq_ids, const int32_t *d_tokens,
                                    int32_t *d_next, void *stream) {
  if (!d || !h_seq_ids || !d_tokens) return set_error(d ? d->ctx : nullptr, VXB_EINVAL, "vxb_decoder_step_device: null argument");
  cudaStream_t user = (cudaStream_t)stream;
  cudaEvent_t ev;
  VXB_CUDA_TRY(d->ctx, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  cudaEventRecord(ev, user);
  cudaStreamWaitEvent(d->stream, ev, 0);
  int rc = launch_step(d, batch, h_seq_ids, d_tokens, false, nullptr);
  if (!rc && d_next)
    rc = cudaMemcpyAsync(d_next, d->d_next, batch * sizeof(int32_t), cudaMemcpyDeviceToDevice, d->stream) == cudaSuccess
             ? VXB_OK : set_error(d->ctx, VXB_ECUDA, "vxb_decoder_step_device: copy of next tokens");
  cudaEventRecord(ev, d->stream);
  cudaStreamWaitEvent(user, ev, 0);
  cudaEventDestroy(ev);
  return rc;
}

// Logits [batch, vocab] of the last step. With tensor parallelism this is a
// collective: every rank calls it, the vocabulary shards are all-gathered.
VXB_API int vxb_decoder_logits(vxb_decoder *d, int batch, float *d_out, void *stream) {
  if (!d || !d_out) return set_error(d ? d->ctx : nullptr, VXB_EINVAL, "vxb_decoder_logits: null argument");
  if (batch < 1 || batch > d->cfg.max_batch) return set_error(d->ctx, VXB_EINVAL, "vxb_decoder_logits: batch %d", batch);
  if (int rc = use_device(d->ctx)) return rc;
  const float *src = d->logits;
  if (d->tp > 1) {
    if (int rc = comm_allgather_f32(d->comm, d->logits, d->logits_all, (size_t)batch * d->vocab, d->stream)) return rc;
    if (int rc = unshard_launch(d->ctx, d->logits_all, d->tp, batch, d->vocab, d->logits_full, d->stream)) return rc;
    src = d->logits_full;
  }
  VXB_CUDA_TRY(d->ctx, cudaStreamSynchronize(d->stream));
  VXB_CUDA_TRY(d->ctx, cudaMemcpyAsync(d_out, src, (size_t)batch * d->cfg.vocab_size * 4, cudaMemcpyDeviceToDevice,
                                       (cudaStream_t)stream));
  return VXB_OK;
}

VXB_API int vxb_decoder_fork(vxb_decoder *d, int64_t src_seq, int64_t dst_seq, int64_t n_tokens) {
  if (!d) return set_error(nullptr, VXB_EINVAL, "vxb_decoder_fork: null decoder");
  if (int rc = use_device(d->ctx)) return rc;
  if (int rc = vxb_kv_fork(d->kv, src_seq, dst_seq, n_tokens, d->stream)) return rc;
  VXB_CUDA_TRY(d->ctx, cudaStreamSynchronize(d->stream));
  return VXB_OK;
}

VXB_API int vxb_decoder_free_seq(vxb_decoder *d, int64_t seq_id) {
  if (!d) return set_error(nullptr, VXB_EINVAL, "vxb_decoder_free_seq: null decoder");
  VXB_CUDA_TRY(d->ctx, cudaStreamSynchronize(d->stream));
  return vxb_kv_free_seq(d->kv, seq_id);
}

VXB_API int vxb_decoder_kv(vxb_decoder *d, vxb_kv **out) {
  if (!d || !out) return set_error(nullptr, VXB_EINVAL, "vxb_decoder_kv: null argument");
  *out = d->kv;
  return VXB_OK;
}

VXB_API int vxb_decoder_stream(vxb_decoder *d, void **out) {
  if (!d || !out) return set_error(nullptr, VXB_EINVAL, "vxb_decoder_stream: null argument");
  *out = (void *)d->stream;
  return VXB_OK;
}
