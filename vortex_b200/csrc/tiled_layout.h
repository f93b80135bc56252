// Geometry of the tiled weight layout (HBM format of a quantized W [N, K]).
//
//   [0, 256)            header: u32 magic, u32 flags, u32 fmt, u32 N, u32 K
//   codes               per 16-row tile t, per k-chunk c (64 K for Q4_0, 32 K for
//                       Q8_0), per lane l: 16 bytes = 512 contiguous bytes per
//                       (t, c). Each 16-byte lane slice holds that lane's
//                       m16n8k16 A-operand fragments: Q4_0 -> 4 u32, one per
//                       k16 step, nibbles (value = code + 8) at bit positions
//                       a0@0 a2@4 a4@8 a6@12 a1@16 a3@20 a5@24 a7@28;
//                       Q8_0 -> 2 u32 per k16 step, int8 codes a0..a3 | a4..a7.
//                       (a_i as in the PTX fragment layout: a0/a1 row g, a2/a3
//                       row g+8, a4..a7 the same rows, with g = lane/4.) The
//                       k order inside a step is permuted: the fragment columns
//                       {2q, 2q+1, 2q+8, 2q+9} of lane q (q = lane%4) hold the
//                       matrix columns {4q, 4q+1, 4q+2, 4q+3}, so the lane's
//                       activation operand is 8 contiguous bytes of x.
//   scales              per tile t, per chunk c, per row pair i (0..7), per
//                       block of the chunk: u32 = f16 scale of row 16t+i (low
//                       half) | row 16t+i+8 (high half).
// Rows beyond N and columns beyond K are padding with code 0 and scale 0.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "../../include/vxb.h"

#define TILED_MAGIC 0x54425856u /* "VXBT" */
#define TILED_FLAG_SUBNORMAL_SCALES 1u

struct TiledGeom {
  int fmt, N, K, N_pad, K_pad, n_tiles, n_chunks, n_blocks, chunk;
  size_t codes_off, codes_bytes, scales_bytes, total_bytes;
};

static inline TiledGeom tiled_geom(int fmt, int N, int K) {
  TiledGeom g;
  g.fmt = fmt;
  g.N = N;
  g.K = K;
  g.chunk = fmt == VXB_Q4_0 ? 64 : 32;
  g.N_pad = (N + 15) / 16 * 16;
  g.K_pad = (K + g.chunk - 1) / g.chunk * g.chunk;
  g.n_tiles = g.N_pad / 16;
  g.n_chunks = g.K_pad / g.chunk;
  g.n_blocks = g.K_pad / 32;
  g.codes_off = 256;
  g.codes_bytes = (size_t)g.n_tiles * g.n_chunks * 512;
  g.scales_bytes = (size_t)g.n_tiles * g.n_blocks * 32;
  g.total_bytes = (g.codes_off + g.codes_bytes + g.scales_bytes + 255) / 256 * 256;
  return g;
}
