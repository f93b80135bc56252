// Geometry of the tiled weight layout (HBM format of a quantized W [N, K]).
//
//   [0, 256)            header: u32 magic, u32 flags, u32 fmt, u32 N, u32 K
//   units               one per (16-row tile t, k-chunk c), stored [t][c], so
//                       the whole k range of one tile is one contiguous
//                       stream. A chunk is 64 columns (Q4_0) or 32 columns
//                       (Q8_0). A unit is
//                         512 bytes of codes, then
//                         8*BPC u32 of scales (BPC = 32-column blocks per chunk).
//   codes of a unit     32 lanes x 16 bytes. Each 16-byte lane slice holds the
//                       lane's m16n8k16 A-operand fragments: Q4_0 -> 4 u32, one
//                       per k16 step, nibbles (value = code + 8) at bit
//                       positions a0@0 a2@4 a4@8 a6@12 a1@16 a3@20 a5@24 a7@28;
//                       Q8_0 -> 2 u32 per k16 step, int8 codes a0..a3 | a4..a7.
//                       (a_i as in the PTX fragment layout: a0/a1 row g, a2/a3
//                       row g+8, a4..a7 the same rows, with g = lane/4.) The k
//                       order inside a step is permuted: the fragment columns
//                       {2q, 2q+1, 2q+8, 2q+9} of lane q (q = lane%4) hold the
//                       matrix columns {4q, 4q+1, 4q+2, 4q+3}, so the lane's
//                       activation operand is 8 contiguous bytes of x.
//   scales of a unit    per row pair i (0..7), per block of the chunk: u32 =
//                       f16 scale of row 16t+i (low half) | row 16t+i+8 (high).
// Rows beyond N (up to a multiple of 128) and columns beyond K (up to a
// multiple of TILED_STAGE_CHUNKS chunks: 256 for Q4_0, 128 for Q8_0) are
// padding with scale 0.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "../../include/vxb.h"

#define TILED_MAGIC 0x54425856u /* "VXBT" */
#define TILED_FLAG_SUBNORMAL_SCALES 1u
#define TILED_STAGE_CHUNKS 4 /* the chunk count is a multiple of this */

#ifdef __CUDACC__
#define TILED_HD __host__ __device__
#else
#define TILED_HD
#endif

struct TiledGeom {
  int fmt, N, K, N_pad, K_pad, n_tiles, n_groups, n_chunks, n_blocks, chunk, bpc;
  size_t codes_off;    // start of the units
  size_t sc_per_tile;  // scale bytes of one unit
  size_t unit;         // bytes of one (tile, chunk) unit: 512 + sc_per_tile
  size_t total_bytes;
};

TILED_HD static inline TiledGeom tiled_geom(int fmt, int N, int K) {
  TiledGeom g;
  g.fmt = fmt;
  g.N = N;
  g.K = K;
  g.chunk = fmt == VXB_Q4_0 ? 64 : 32;
  g.bpc = g.chunk / 32;
  g.N_pad = (N + 127) / 128 * 128;
  const int span = g.chunk * TILED_STAGE_CHUNKS;
  g.K_pad = (K + span - 1) / span * span;
  g.n_tiles = g.N_pad / 16;
  g.n_groups = g.N_pad / 128;
  g.n_chunks = g.K_pad / g.chunk;
  g.n_blocks = g.K_pad / 32;
  g.codes_off = 256;
  g.sc_per_tile = (size_t)8 * g.bpc * 4;
  g.unit = 512 + g.sc_per_tile;
  g.total_bytes = (g.codes_off + (size_t)g.n_tiles * g.n_chunks * g.unit + 255) / 256 * 256;
  return g;
}

// byte offset of the unit (codes, lane slices follow) of tile t, chunk c
TILED_HD static inline size_t tiled_codes_at(const TiledGeom &g, int t, int c) {
  return g.codes_off + ((size_t)t * g.n_chunks + c) * g.unit;
}

// byte offset of the scales of tile t, chunk c
TILED_HD static inline size_t tiled_scales_at(const TiledGeom &g, int t, int c) {
  return tiled_codes_at(g, t, c) + 512;
}
