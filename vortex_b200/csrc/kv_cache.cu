// Paged KV cache on the device.
//
// Follows PagedKVCache (src/kv_cache.rs:29-93): a fixed pool of max_blocks
// blocks of block_size tokens, a block table per (layer, seq_id), a free-block
// stack initialised to (0..max_blocks).rev() so blocks are handed out 0, 1, 2,
// ...; append_kv pops a block when the sequence's last block is full;
// free_seq returns every block of the sequence (all layers) to the stack.
// The reference stores one f64 vector per token and never uses num_heads; here
// a token holds [num_kv_heads, head_dim] keys and values in bf16, or int8 with
// one f32 scale per (token, head) computed by calibrate_minmax
// (src/quantize.rs:585-591: absmax/127, all-zero -> 1.0) and codes
// round-half-away(v/scale) clamped to [-128, 127] (src/quantize.rs:105-108).
#include <algorithm>
#include <cmath>

#include "kv_cache.h"

using namespace vxb;

namespace {

__device__ __forceinline__ void append_token(const KVPlace &p, int i, int layer, int H, int D, int bs, int max_seqs,
                                             int mbps, int is_int8, const uint16_t *__restrict__ k,
                                             const uint16_t *__restrict__ v, void *pool_k, void *pool_v,
                                             float *scale_k, float *scale_v, int32_t *tables, int32_t *lens) {
  const size_t row = (size_t)H * D;
  if (!is_int8) {
    // 16-byte pieces of the token's [H, D] keys and values
    const int pieces = (int)(row / 8);
    for (int c = threadIdx.x; c < 2 * pieces; c += blockDim.x) {
      const bool isv = c >= pieces;
      const int cc = isv ? c - pieces : c;
      const int h = (cc * 8) / D, dd = (cc * 8) % D;
      const uint4 val = *reinterpret_cast<const uint4 *>((isv ? v : k) + (size_t)i * row + (size_t)cc * 8);
      uint16_t *dst = reinterpret_cast<uint16_t *>(isv ? pool_v : pool_k) +
                      (((size_t)p.block * H + h) * bs + p.offset) * D + dd;
      *reinterpret_cast<uint4 *>(dst) = val;
    }
  } else {
    // one warp per (head, k|v) row: f64 absmax/127 scale, round-half-away codes
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int r = warp; r < 2 * H; r += nw) {
      const bool isv = r >= H;
      const int h = isv ? r - H : r;
      const uint16_t *src = (isv ? v : k) + (size_t)i * row + (size_t)h * D;
      double m = 0.0;
      for (int dd = lane; dd < D; dd += 32) m = fmax(m, fabs((double)bf16_bits_to_f32(src[dd])));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
      const double scale = m == 0.0 ? 1.0 : m / 127.0;
      int8_t *dst = reinterpret_cast<int8_t *>(isv ? pool_v : pool_k) + (((size_t)p.block * H + h) * bs + p.offset) * D;
      for (int dd = lane; dd < D; dd += 32) {
        const double q = round((double)bf16_bits_to_f32(src[dd]) / scale);
        dst[dd] = (int8_t)(isnan(q) ? 0.0 : fmin(fmax(q, -128.0), 127.0));
      }
      if (lane == 0) (isv ? scale_v : scale_k)[((size_t)p.block * H + h) * bs + p.offset] = (float)scale;
    }
  }
  if (threadIdx.x == 0) {
    if (p.offset == 0) tables[((size_t)layer * max_seqs + p.slot) * mbps + p.pos / bs] = p.block;
    atomicMax(lens + (size_t)layer * max_seqs + p.slot, p.pos + 1);
  }
}

__global__ void kv_append_kernel(const KVPlace *__restrict__ places, int layer, int H, int D, int bs, int max_seqs,
                                 int mbps, int is_int8, const uint16_t *__restrict__ k, const uint16_t *__restrict__ v,
                                 void *pool_k, void *pool_v, float *scale_k, float *scale_v, int32_t *tables,
                                 int32_t *lens) {
  const int i = blockIdx.x;
  const KVPlace p = places[i];
  append_token(p, i, layer, H, D, bs, max_seqs, mbps, is_int8, k, v, pool_k, pool_v, scale_k, scale_v, tables, lens);
}

// get_kv (src/kv_cache.rs:69-80) for tests: dequantized f32 [len, H, D].
__global__ void kv_gather_kernel(const int32_t *__restrict__ table, int len, int H, int D, int bs, int is_int8,
                                 const void *pool_k, const void *pool_v, const float *scale_k, const float *scale_v,
                                 float *__restrict__ k_out, float *__restrict__ v_out) {
  const int pos = blockIdx.x;
  if (pos >= len) return;
  const int block = table[pos / bs], off = pos % bs;
  for (int e = threadIdx.x; e < H * D; e += blockDim.x) {
    const int h = e / D, dd = e % D;
    const size_t idx = (((size_t)block * H + h) * bs + off) * D + dd;
    const size_t o = (size_t)pos * H * D + e;
    if (!is_int8) {
      k_out[o] = bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(pool_k)[idx]);
      v_out[o] = bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(pool_v)[idx]);
    } else {
      const size_t si = ((size_t)block * H + h) * bs + off;
      k_out[o] = (float)reinterpret_cast<const int8_t *>(pool_k)[idx] * scale_k[si];
      v_out[o] = (float)reinterpret_cast<const int8_t *>(pool_v)[idx] * scale_v[si];
    }
  }
}

// The first `rows` token rows of every head of block `src` into block `dst`
// (keys, values and, for int8, their scales): the private copy of a forked
// sequence's partly filled last block.
__global__ void kv_copy_rows_kernel(uint8_t *pool_k, uint8_t *pool_v, float *scale_k, float *scale_v, int src, int dst,
                                    int H, int bs, int D, int elem, int rows) {
  const int h = blockIdx.x;
  const size_t row_bytes = (size_t)D * elem;
  const size_t so = ((size_t)src * H + h) * bs * row_bytes, d0 = ((size_t)dst * H + h) * bs * row_bytes;
  const size_t n = (size_t)rows * row_bytes;
  for (size_t i = threadIdx.x * 4; i < n; i += (size_t)blockDim.x * 4) {
    *reinterpret_cast<uint32_t *>(pool_k + d0 + i) = *reinterpret_cast<const uint32_t *>(pool_k + so + i);
    *reinterpret_cast<uint32_t *>(pool_v + d0 + i) = *reinterpret_cast<const uint32_t *>(pool_v + so + i);
  }
  if (scale_k)
    for (int r = threadIdx.x; r < rows; r += blockDim.x) {
      scale_k[((size_t)dst * H + h) * bs + r] = scale_k[((size_t)src * H + h) * bs + r];
      scale_v[((size_t)dst * H + h) * bs + r] = scale_v[((size_t)src * H + h) * bs + r];
    }
}

int kv_check(vxb_kv *kv, const char *who) {
  if (!kv || !kv->ctx) return set_error(nullptr, VXB_EINVAL, "%s: null cache", who);
  return VXB_OK;
}

}  // namespace

namespace vxb {

int kv_place(vxb_kv *kv, int layer, int64_t seq_id, KVPlace *out) {
  auto key = std::make_pair(layer, seq_id);
  auto it = kv->tables.find(key);
  int slot;
  auto si = kv->slot_of.find(seq_id);
  if (si == kv->slot_of.end()) {
    if (kv->free_slots.empty())
      return set_error(kv->ctx, VXB_ENOBLOCKS, "KV cache has no free sequence slot (max_seqs=%d)", kv->max_seqs);
    slot = kv->free_slots.back();
    kv->free_slots.pop_back();
    kv->slot_of[seq_id] = slot;
  } else {
    slot = si->second;
  }
  vxb_kv::Table &t = it == kv->tables.end() ? kv->tables[key] : it->second;
  const bool needs_block = t.blocks.empty() || t.len % kv->block_size == 0;
  if (needs_block) {
    if ((int)t.blocks.size() >= kv->max_blocks_per_seq)
      return set_error(kv->ctx, VXB_ENOBLOCKS, "sequence %lld exceeds max_blocks_per_seq=%d", (long long)seq_id,
                       kv->max_blocks_per_seq);
    if (kv->free_blocks.empty()) return set_error(kv->ctx, VXB_ENOBLOCKS, "KV cache out of blocks");
    t.blocks.push_back(kv->free_blocks.back());
    kv->refs[kv->free_blocks.back()] = 1;
    kv->free_blocks.pop_back();
  }
  out->block = t.blocks.back();
  out->offset = (int32_t)(t.len % kv->block_size);
  out->slot = slot;
  out->pos = (int32_t)t.len;
  t.len++;
  return VXB_OK;
}

void kv_release_block(vxb_kv *kv, int32_t b) {
  if (--kv->refs[b] <= 0) {
    kv->refs[b] = 0;
    kv->free_blocks.push_back(b);
  }
}

void kv_unplace(vxb_kv *kv, int layer, int64_t seq_id, int n) {
  auto it = kv->tables.find(std::make_pair(layer, seq_id));
  if (it == kv->tables.end()) return;
  vxb_kv::Table &t = it->second;
  for (int i = 0; i < n && t.len > 0; i++) {
    t.len--;
    if (t.len % kv->block_size == 0 && !t.blocks.empty()) {
      kv_release_block(kv, t.blocks.back());
      t.blocks.pop_back();
    }
  }
}

int kv_append_launch(vxb_kv *kv, int layer, int n, const KVPlace *d_places, const uint16_t *d_k, const uint16_t *d_v,
                     cudaStream_t st) {
  if (n <= 0) return VXB_OK;
  kv_append_kernel<<<n, 128, 0, st>>>(d_places, layer, kv->num_kv_heads, kv->head_dim, kv->block_size, kv->max_seqs,
                                      kv->max_blocks_per_seq, kv->dtype == VXB_I8, d_k, d_v, kv->pool_k, kv->pool_v,
                                      kv->scale_k, kv->scale_v, kv->d_tables, kv->d_lens);
  return launch_check(kv->ctx, "kv_append_kernel");
}

}  // namespace vxb

VXB_API int vxb_kv_create(vxb_ctx *ctx, int num_layers, int num_kv_heads, int head_dim, int block_size,
                          int max_blocks, int max_seqs, int max_blocks_per_seq, int kv_dtype, vxb_kv **out) {
  if (!ctx || !out) return set_error(ctx, VXB_EINVAL, "vxb_kv_create: null argument");
  *out = nullptr;
  if (num_layers <= 0 || num_kv_heads <= 0 || max_blocks <= 0 || max_seqs <= 0 || max_blocks_per_seq <= 0)
    return set_error(ctx, VXB_EINVAL, "vxb_kv_create: sizes must be positive");
  if (head_dim != 64 && head_dim != 128)
    return set_error(ctx, VXB_EUNSUPPORTED, "vxb_kv_create: head_dim %d (supported: 64, 128)", head_dim);
  if (block_size <= 0 || block_size % 16)
    return set_error(ctx, VXB_EINVAL, "vxb_kv_create: block_size %d must be a positive multiple of 16", block_size);
  if (kv_dtype != VXB_BF16 && kv_dtype != VXB_I8)
    return set_error(ctx, VXB_EINVAL, "vxb_kv_create: kv_dtype must be VXB_BF16 or VXB_I8");
  if (int rc = use_device(ctx)) return rc;
  vxb_kv *kv = new vxb_kv();
  kv->ctx = ctx;
  kv->num_layers = num_layers;
  kv->num_kv_heads = num_kv_heads;
  kv->head_dim = head_dim;
  kv->block_size = block_size;
  kv->max_blocks = max_blocks;
  kv->max_seqs = max_seqs;
  kv->max_blocks_per_seq = max_blocks_per_seq;
  kv->dtype = kv_dtype;
  kv->elem_bytes = kv_dtype == VXB_I8 ? 1 : 2;
  const size_t pool = (size_t)max_blocks * num_kv_heads * block_size * head_dim * kv->elem_bytes;
  const size_t tbl = (size_t)num_layers * max_seqs * max_blocks_per_seq * sizeof(int32_t);
  const size_t lens = (size_t)num_layers * max_seqs * sizeof(int32_t);
  bool ok = cudaMalloc(&kv->pool_k, pool) == cudaSuccess && cudaMalloc(&kv->pool_v, pool) == cudaSuccess &&
            cudaMalloc((void **)&kv->d_tables, tbl) == cudaSuccess && cudaMalloc((void **)&kv->d_lens, lens) == cudaSuccess;
  if (ok && kv_dtype == VXB_I8) {
    const size_t sc = (size_t)max_blocks * num_kv_heads * block_size * sizeof(float);
    ok = cudaMalloc((void **)&kv->scale_k, sc) == cudaSuccess && cudaMalloc((void **)&kv->scale_v, sc) == cudaSuccess;
  }
  if (ok) ok = cudaMemset(kv->d_tables, 0xFF, tbl) == cudaSuccess && cudaMemset(kv->d_lens, 0, lens) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    vxb_kv_destroy(kv);
    return set_error(ctx, VXB_ENOMEM, "vxb_kv_create: device allocation failed (pool %zu bytes x2)", pool);
  }
  kv->free_blocks.reserve(max_blocks);
  for (int b = max_blocks - 1; b >= 0; b--) kv->free_blocks.push_back(b);
  kv->refs.assign(max_blocks, 0);
  for (int s = max_seqs - 1; s >= 0; s--) kv->free_slots.push_back(s);
  *out = kv;
  return VXB_OK;
}

VXB_API int vxb_kv_destroy(vxb_kv *kv) {
  if (!kv) return VXB_OK;
  if (kv->ctx) use_device(kv->ctx);
  cudaFree(kv->pool_k);
  cudaFree(kv->pool_v);
  cudaFree(kv->scale_k);
  cudaFree(kv->scale_v);
  cudaFree(kv->d_tables);
  cudaFree(kv->d_lens);
  delete kv;
  return VXB_OK;
}

static int upload_places(vxb_kv *kv, const std::vector<KVPlace> &pl, cudaStream_t st, KVPlace **d_out) {
  const size_t bytes = pl.size() * sizeof(KVPlace);
  if (int rc = ws_reserve(kv->ctx, bytes, 0)) return rc;
  VXB_CUDA_TRY(kv->ctx, cudaMemcpyAsync(kv->ctx->ws, pl.data(), bytes, cudaMemcpyHostToDevice, st));
  *d_out = (KVPlace *)kv->ctx->ws;
  return VXB_OK;
}

VXB_API int vxb_kv_append(vxb_kv *kv, int layer, int n, const int64_t *h_seq_ids, const uint16_t *d_k,
                          const uint16_t *d_v, void *stream) {
  if (int rc = kv_check(kv, "vxb_kv_append")) return rc;
  if (layer < 0 || layer >= kv->num_layers) return set_error(kv->ctx, VXB_EINVAL, "vxb_kv_append: layer %d out of range", layer);
  if (n < 0 || (n > 0 && (!h_seq_ids || !d_k || !d_v))) return set_error(kv->ctx, VXB_EINVAL, "vxb_kv_append: bad arguments");
  if (n == 0) return VXB_OK;
  for (int i = 0; i < n; i++)
    for (int j = 0; j < i; j++)
      if (h_seq_ids[i] == h_seq_ids[j])
        return set_error(kv->ctx, VXB_EINVAL, "vxb_kv_append: sequence %lld listed twice", (long long)h_seq_ids[i]);
  if (int rc = use_device(kv->ctx)) return rc;
  std::vector<KVPlace> pl(n);
  for (int i = 0; i < n; i++) {
    if (int rc = kv_place(kv, layer, h_seq_ids[i], &pl[i])) {
      for (int j = i - 1; j >= 0; j--) kv_unplace(kv, layer, h_seq_ids[j], 1);
      return rc;
    }
  }
  KVPlace *d_pl = nullptr;
  cudaStream_t st = (cudaStream_t)stream;
  if (int rc = upload_places(kv, pl, st, &d_pl)) return rc;
  return kv_append_launch(kv, layer, n, d_pl, d_k, d_v, st);
}

VXB_API int vxb_kv_append_seq(vxb_kv *kv, int layer, int64_t seq_id, int n_tokens, const uint16_t *d_k,
                              const uint16_t *d_v, void *stream) {
  if (int rc = kv_check(kv, "vxb_kv_append_seq")) return rc;
  if (layer < 0 || layer >= kv->num_layers) return set_error(kv->ctx, VXB_EINVAL, "vxb_kv_append_seq: layer out of range");
  if (n_tokens < 0 || (n_tokens > 0 && (!d_k || !d_v))) return set_error(kv->ctx, VXB_EINVAL, "vxb_kv_append_seq: bad arguments");
  if (n_tokens == 0) return VXB_OK;
  if (int rc = use_device(kv->ctx)) return rc;
  std::vector<KVPlace> pl(n_tokens);
  for (int i = 0; i < n_tokens; i++) {
    if (int rc = kv_place(kv, layer, seq_id, &pl[i])) {
      kv_unplace(kv, layer, seq_id, i);
      return rc;
    }
  }
  KVPlace *d_pl = nullptr;
  cudaStream_t st = (cudaStream_t)stream;
  if (int rc = upload_places(kv, pl, st, &d_pl)) return rc;
  return kv_append_launch(kv, layer, n_tokens, d_pl, d_k, d_v, st);
}

VXB_API int vxb_kv_free_seq(vxb_kv *kv, int64_t seq_id) {
  if (int rc = kv_check(kv, "vxb_kv_free_seq")) return rc;
  bool any = false;
  for (int layer = 0; layer < kv->num_layers; layer++) {
    auto it = kv->tables.find(std::make_pair(layer, seq_id));
    if (it == kv->tables.end()) continue;
    any = true;
    for (int32_t b : it->second.blocks) kv_release_block(kv, b);
    kv->tables.erase(it);
  }
  auto si = kv->slot_of.find(seq_id);
  if (si != kv->slot_of.end()) {
    const int slot = si->second;
    kv->free_slots.push_back(slot);
    kv->slot_of.erase(si);
    if (int rc = use_device(kv->ctx)) return rc;
    // lengths of the freed slot go back to zero (tables are rewritten on reuse)
    for (int layer = 0; layer < kv->num_layers; layer++)
      VXB_CUDA_TRY(kv->ctx, cudaMemsetAsync(kv->d_lens + (size_t)layer * kv->max_seqs + slot, 0, sizeof(int32_t), 0));
    VXB_CUDA_TRY(kv->ctx, cudaStreamSynchronize(0));
  }
  (void)any;
  return VXB_OK;
}

VXB_API int vxb_kv_stats(const vxb_kv *kv, int64_t *out6) {
  if (!kv || !out6) return set_error(nullptr, VXB_EINVAL, "vxb_kv_stats: null argument");
  out6[0] = kv->max_blocks - (int64_t)kv->free_blocks.size();  // used_blocks
  out6[1] = (int64_t)kv->free_blocks.size();                   // free_blocks
  out6[2] = kv->block_size;                                    // block_size
  out6[3] = (int64_t)kv->tables.size();                        // num_seqs (tables, as the reference counts)
  out6[4] = out6[0] * kv->num_kv_heads * kv->block_size * kv->head_dim * (int64_t)kv->elem_bytes * 2;  // device bytes
  out6[5] = (int64_t)kv->slot_of.size();                       // distinct sequences
  return VXB_OK;
}

VXB_API int vxb_kv_seq_len(const vxb_kv *kv, int layer, int64_t seq_id, int64_t *len) {
  if (!kv || !len) return set_error(nullptr, VXB_EINVAL, "vxb_kv_seq_len: null argument");
  auto it = kv->tables.find(std::make_pair(layer, seq_id));
  *len = it == kv->tables.end() ? 0 : it->second.len;
  return VXB_OK;
}

VXB_API int vxb_kv_block_table(const vxb_kv *kv, int layer, int64_t seq_id, int32_t *h_out, int cap, int *n) {
  if (!kv || !n) return set_error(nullptr, VXB_EINVAL, "vxb_kv_block_table: null argument");
  auto it = kv->tables.find(std::make_pair(layer, seq_id));
  *n = it == kv->tables.end() ? 0 : (int)it->second.blocks.size();
  if (it != kv->tables.end() && h_out)
    for (int i = 0; i < *n && i < cap; i++) h_out[i] = it->second.blocks[i];
  return VXB_OK;
}

VXB_API int vxb_kv_gather(vxb_kv *kv, int layer, int64_t seq_id, float *d_k_out, float *d_v_out, void *stream) {
  if (int rc = kv_check(kv, "vxb_kv_gather")) return rc;
  auto it = kv->tables.find(std::make_pair(layer, seq_id));
  if (it == kv->tables.end() || it->second.len == 0) return VXB_OK;
  if (!d_k_out || !d_v_out) return set_error(kv->ctx, VXB_EINVAL, "vxb_kv_gather: null output");
  if (int rc = use_device(kv->ctx)) return rc;
  const int slot = kv->slot_of.at(seq_id);
  const int32_t *table = kv->d_tables + ((size_t)layer * kv->max_seqs + slot) * kv->max_blocks_per_seq;
  kv_gather_kernel<<<(unsigned)it->second.len, 128, 0, (cudaStream_t)stream>>>(
      table, (int)it->second.len, kv->num_kv_heads, kv->head_dim, kv->block_size, kv->dtype == VXB_I8, kv->pool_k,
      kv->pool_v, kv->scale_k, kv->scale_v, d_k_out, d_v_out);
  return launch_check(kv->ctx, "kv_gather_kernel");
}

// Prefix reuse: sequence dst_seq starts as the first n_tokens tokens of
// src_seq in every layer. Full blocks are shared (each block counts the
// tables holding it; a shared block is never written again: appends go to
// a sequence's own last block or to a new one), a partly filled last block is
// copied into a block of dst's own. The reference only declares a
// prefix_cache map (src/kv_cache.rs:37, 44) and never fills it.
VXB_API int vxb_kv_fork(vxb_kv *kv, int64_t src_seq, int64_t dst_seq, int64_t n_tokens, void *stream) {
  if (int rc = kv_check(kv, "vxb_kv_fork")) return rc;
  if (src_seq == dst_seq) return set_error(kv->ctx, VXB_EINVAL, "vxb_kv_fork: source and target are the same sequence");
  if (n_tokens < 0) return set_error(kv->ctx, VXB_EINVAL, "vxb_kv_fork: negative token count");
  for (int l = 0; l < kv->num_layers; l++) {
    auto d = kv->tables.find(std::make_pair(l, dst_seq));
    if (d != kv->tables.end() && d->second.len > 0)
      return set_error(kv->ctx, VXB_EINVAL, "vxb_kv_fork: sequence %lld already holds tokens", (long long)dst_seq);
    auto sit = kv->tables.find(std::make_pair(l, src_seq));
    const int64_t have = sit == kv->tables.end() ? 0 : sit->second.len;
    if (n_tokens > have)
      return set_error(kv->ctx, VXB_EINVAL, "vxb_kv_fork: sequence %lld holds %lld tokens in layer %d, %lld asked",
                       (long long)src_seq, (long long)have, l, (long long)n_tokens);
  }
  if (n_tokens == 0) return VXB_OK;
  const int bs = kv->block_size;
  const int64_t full = n_tokens / bs, rem = n_tokens % bs;
  if (full + (rem > 0) > kv->max_blocks_per_seq)
    return set_error(kv->ctx, VXB_ENOBLOCKS, "sequence %lld exceeds max_blocks_per_seq=%d", (long long)dst_seq,
                     kv->max_blocks_per_seq);
  if (rem > 0 && (int64_t)kv->free_blocks.size() < kv->num_layers)
    return set_error(kv->ctx, VXB_ENOBLOCKS, "KV cache out of blocks");
  int slot;
  auto si = kv->slot_of.find(dst_seq);
  if (si == kv->slot_of.end()) {
    if (kv->free_slots.empty())
      return set_error(kv->ctx, VXB_ENOBLOCKS, "KV cache has no free sequence slot (max_seqs=%d)", kv->max_seqs);
    slot = kv->free_slots.back();
    kv->free_slots.pop_back();
    kv->slot_of[dst_seq] = slot;
  } else {
    slot = si->second;
  }
  if (int rc = use_device(kv->ctx)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  std::vector<int32_t> tab;
  for (int l = 0; l < kv->num_layers; l++) {
    const vxb_kv::Table &s = kv->tables.at(std::make_pair(l, src_seq));
    vxb_kv::Table &t = kv->tables[std::make_pair(l, dst_seq)];
    t.blocks.assign(s.blocks.begin(), s.blocks.begin() + full);
    for (int32_t b : t.blocks) kv->refs[b]++;
    if (rem > 0) {
      const int32_t b = kv->free_blocks.back();
      kv->free_blocks.pop_back();
      kv->refs[b] = 1;
      kv_copy_rows_kernel<<<kv->num_kv_heads, 256, 0, st>>>(
          (uint8_t *)kv->pool_k, (uint8_t *)kv->pool_v, kv->scale_k, kv->scale_v, s.blocks[full], b, kv->num_kv_heads,
          bs, kv->head_dim, (int)kv->elem_bytes, (int)rem);
      if (int rc = launch_check(kv->ctx, "kv_copy_rows_kernel")) return rc;
      t.blocks.push_back(b);
    }
    t.len = n_tokens;
    tab = t.blocks;
    const size_t row = ((size_t)l * kv->max_seqs + slot);
    VXB_CUDA_TRY(kv->ctx, cudaMemcpyAsync(kv->d_tables + row * kv->max_blocks_per_seq, tab.data(),
                                          tab.size() * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    const int32_t len = (int32_t)n_tokens;
    VXB_CUDA_TRY(kv->ctx, cudaMemcpyAsync(kv->d_lens + row, &len, sizeof(int32_t), cudaMemcpyHostToDevice, st));
    VXB_CUDA_TRY(kv->ctx, cudaStreamSynchronize(st));  // tab and len are host temporaries
  }
  return VXB_OK;
}
