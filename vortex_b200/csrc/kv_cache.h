// Paged KV cache: host-side block allocator (PagedKVCache semantics) plus the
// device pools the attention kernels read.
#pragma once

#include <map>
#include <unordered_map>
#include <vector>

#include "vxb_internal.h"

// One token's placement, consumed by the append kernel.
struct KVPlace {
  int32_t block;   // pool block id
  int32_t offset;  // token offset inside the block
  int32_t slot;    // sequence slot of the device block table
  int32_t pos;     // token index within the sequence (= length before append)
};

struct vxb_kv {
  vxb_ctx *ctx = nullptr;
  int num_layers = 0, num_kv_heads = 0, head_dim = 0, block_size = 0, max_blocks = 0;
  int max_seqs = 0, max_blocks_per_seq = 0, dtype = VXB_BF16;
  size_t elem_bytes = 2;
  // device pools: [max_blocks][H][block_size][head_dim] (bf16 or int8)
  void *pool_k = nullptr, *pool_v = nullptr;
  // int8 only: per-(block, head, token) f32 scales [max_blocks][H][block_size]
  float *scale_k = nullptr, *scale_v = nullptr;
  // device block tables [num_layers][max_seqs][max_blocks_per_seq] and lengths [num_layers][max_seqs]
  int32_t *d_tables = nullptr, *d_lens = nullptr;
  // host mirror
  struct Table {
    std::vector<int32_t> blocks;
    int64_t len = 0;
  };
  std::map<std::pair<int, int64_t>, Table> tables;  // (layer, seq_id) -> table
  std::vector<int32_t> free_blocks;                   // stack; back() is popped next
  std::vector<int32_t> refs;                          // tables holding each block (a fork shares blocks)
  std::unordered_map<int64_t, int> slot_of;           // seq_id -> slot
  std::vector<int> free_slots;                        // stack of unused slots
};

namespace vxb {

// Reserve placement for one appended token of (layer, seq_id): pops a block
// from the free stack when the sequence's last block is full
// (PagedKVCache::append_kv, src/kv_cache.rs:54-67).
int kv_place(vxb_kv *kv, int layer, int64_t seq_id, KVPlace *out);

// Drop one table's hold on a block; the block returns to the free stack when
// no table holds it.
void kv_release_block(vxb_kv *kv, int32_t b);

// Roll back the placements of a failed multi-token append.
void kv_unplace(vxb_kv *kv, int layer, int64_t seq_id, int n);

// Launch the append kernel for n placements stored in device memory
// (d_places) with keys/values [n, H, d] bf16.
int kv_append_launch(vxb_kv *kv, int layer, int n, const KVPlace *d_places, const uint16_t *d_k,
                     const uint16_t *d_v, cudaStream_t st);

}  // namespace vxb
