// Internal interface of the K4 decode attention (shared with the decoder).
#pragma once

#include "kv_cache.h"

namespace vxb {

struct DecodePlan {
  int splits;  // token splits per (sequence, kv head)
  int tps;     // tokens per split (multiple of 64)
};

// decode_plan never returns more splits than this
constexpr int kMaxDecodeSplits = 12;

DecodePlan decode_plan(const vxb_ctx *ctx, int n, int Hkv, int max_len);
size_t decode_ws_bytes(int n, int Hkv, int G, int D, int splits);

// Cache slot per query row (-1 = empty sequence).
// ws: device scratch of decode_ws_bytes(...) bytes; counters come from ctx.
// Slot ids come from d_slots (device) or, when it is null, from h_slots
// copied into the kernel parameters (n <= 256).
int decode_attn_launch(vxb_kv *kv, int layer, int n, const int32_t *d_slots, const int32_t *h_slots,
                       const uint16_t *d_q, int Hq, float softmax_scale, uint16_t *d_out, float *d_lse,
                       const DecodePlan &p, float *ws, cudaStream_t st);

}  // namespace vxb
