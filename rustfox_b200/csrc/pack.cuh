// HBM weight layout: GGUF blocks regrouped into 16-byte-aligned planes.
//
// A matrix of n_rows x K (nb blocks per row) is cut into units of U whole
// rows. Inside a unit the U*nb blocks keep their GGUF order (row-major, block
// index fastest) but each block is split into segments and every segment
// gets its own plane: plane s holds segment s of block 0, block 1, ... of the
// unit. Thread t of a GEMV CTA owns block t of the unit, so a warp's load of a
// 16-byte segment is one contiguous 512-byte run. The repack is a pure byte
// permutation: the device holds exactly the GGUF bytes, so every decoded
// value is the one upstream decodes, and the bytes streamed per token are the
// GGUF bytes.
//
// U is chosen so U*nb is a multiple of 8 (every unit starts 16-byte aligned:
// 54, 66, 34 and 210 are 2 mod 4 and 144 is a multiple of 16) and the CTA of
// U*nb threads wastes few lanes.
#pragma once

#include "common.cuh"

namespace fox {

struct Seg { uint8_t src, size; };

// Segments in plane order. Plane p of a unit with `count` blocks starts at
// count * (sum of the sizes of planes before p).
struct SegTable { int n; Seg s[14]; };

__host__ __device__ inline SegTable seg_table(int type) {
  switch (type) {
    case T_TQ1_0:  // qs[0..47] in three 16 B planes, qh[48..51], d[52..53]
      return {5, {{0, 16}, {16, 16}, {32, 16}, {48, 4}, {52, 2}}};
    case T_TQ2_0:  // qs[0..63] in four 16 B planes, d[64..65]
      return {5, {{0, 16}, {16, 16}, {32, 16}, {48, 16}, {64, 2}}};
    case T_Q8_0:   // qs[2..33] in two 16 B planes, then d[0..1]
      return {3, {{2, 16}, {18, 16}, {0, 2}}};
    case T_Q4_K:   // qs[16..143] in eight planes, scales[4..15] as 3 words, d|dmin[0..3]
      return {12, {{16, 16}, {32, 16}, {48, 16}, {64, 16}, {80, 16}, {96, 16}, {112, 16},
                   {128, 16}, {4, 4}, {8, 4}, {12, 4}, {0, 4}}};
    case T_Q6_K:   // ql[0..127] eight planes, qh[128..191] four, scales[192..207], d[208..209]
      return {14, {{0, 16}, {16, 16}, {32, 16}, {48, 16}, {64, 16}, {80, 16}, {96, 16},
                   {112, 16}, {128, 16}, {144, 16}, {160, 16}, {176, 16}, {192, 16},
                   {208, 2}}};
    default:
      return {0, {}};
  }
}

// Rows per unit for nb blocks per row (see file comment). Always even, so
// adjacent row pairs (RoPE) and the two halves of a gate/up unit stay together.
inline int unit_rows(int type, int nb) {
  int best = -1;
  double best_waste = 2.0;
  for (int U = 2; U <= 32; U *= 2) {  // even: RoPE pairs and gate/up halves
    long t = (long)U * nb;
    if (t > ((type == T_Q4_K || type == T_Q6_K) ? 256 : 512)) break;  // gemv CTA cap
    if (type != T_Q4_K && t % 8) continue;
    long padded = (t + 31) / 32 * 32;
    double waste = double(padded - t) / double(padded);
    if (waste <= 0.0625 && t >= 64) return U;
    if (waste < best_waste - 1e-9) { best_waste = waste; best = U; }
  }
  return best;  // -1: no unit fits one CTA (the caller reports it)
}

__global__ void pack_kernel(int type, const uint8_t* __restrict__ src, int n_rows, int nb, int U,
                            uint8_t* __restrict__ dst) {
  const long total = (long)n_rows * nb;
  const int BB = block_bytes(type);
  const SegTable tab = seg_table(type);
  for (long g = blockIdx.x * (long)blockDim.x + threadIdx.x; g < total;
       g += (long)gridDim.x * blockDim.x) {
    const long row = g / nb;
    const int u = (int)(row / U);
    const int ru = min(U, n_rows - u * U);
    const long count = (long)ru * nb;
    const long t = g - (long)u * U * nb;  // block index inside the unit
    const uint8_t* s = src + g * BB;
    uint8_t* base = dst + (long)u * U * nb * BB;
    long plane = 0;
    for (int p = 0; p < tab.n; ++p) {
      const int sz = tab.s[p].size;
      uint8_t* d = base + plane * count + t * sz;
      for (int i = 0; i < sz; ++i) d[i] = s[tab.s[p].src + i];
      plane += sz;
    }
  }
}

// TQ1_0 -> TQ2_0 on the device, one thread per 256 block. The decode
// follows upstream's TQ1_0 rule (src/ternary.c:59-93): the level-l trit of
// byte c is ((c * 3^l mod 256) * 3) >> 8, minus 1, for elements l*32 + m
// (qs[m]), 160 + l*16 + m (qs[32+m]) and 240 + l*4 + m (qh[m]). Each trit + 1
// is written as the 2-bit TQ2_0 code of the same element (bits 2l of
// qs[j*32+m] for element j*128 + l*32 + m, src/ternary.c:177-188), and the
// fp16 scale is copied. Every block's trits and scale are unchanged, so
// every integer block sum, and everything computed from it, is unchanged.
__global__ void tq1_to_tq2_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                  long n_blocks) {
  const long b = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (b >= n_blocks) return;
  const uint8_t* in = src + b * 54;
  uint8_t codes[256];
  const uint8_t pow3[5] = {1, 3, 9, 27, 81};
  for (int l = 0; l < 5; ++l)
    for (int m = 0; m < 32; ++m)
      codes[l * 32 + m] = (uint8_t)(((unsigned)(uint8_t)(in[m] * pow3[l]) * 3u) >> 8);
  for (int l = 0; l < 5; ++l)
    for (int m = 0; m < 16; ++m)
      codes[160 + l * 16 + m] = (uint8_t)(((unsigned)(uint8_t)(in[32 + m] * pow3[l]) * 3u) >> 8);
  for (int l = 0; l < 4; ++l)
    for (int m = 0; m < 4; ++m)
      codes[240 + l * 4 + m] = (uint8_t)(((unsigned)(uint8_t)(in[48 + m] * pow3[l]) * 3u) >> 8);
  uint8_t* out = dst + b * 66;
  for (int j = 0; j < 2; ++j)
    for (int m = 0; m < 32; ++m) {
      unsigned q = 0;
      for (int l = 0; l < 4; ++l) q |= (unsigned)codes[j * 128 + l * 32 + m] << (2 * l);
      out[j * 32 + m] = (uint8_t)q;
    }
  out[64] = in[52];
  out[65] = in[53];
}

// Q8_0 rows for q8_rows_kernel (rows.cuh): units of 32 rows; in a unit,
// block b of row r puts qs[0..16) at plane 0 [b][r], qs[16..32) at plane 1
// [b][r] and d at plane 2 [b][r]. A byte permutation of the GGUF bytes.
__global__ void pack_q8_rows32_kernel(const uint8_t* __restrict__ src, int n_rows, int nb,
                                      uint8_t* __restrict__ dst) {
  const long total = (long)n_rows * nb;
  for (long g = blockIdx.x * (long)blockDim.x + threadIdx.x; g < total;
       g += (long)gridDim.x * blockDim.x) {
    const long row = g / nb;
    const int b = (int)(g - row * nb);
    const long u = row / 32;
    const int r = (int)(row - u * 32);
    const uint8_t* in = src + g * 34;
    uint8_t* base = dst + u * (long)nb * 32 * 34;
    uint8_t* p0 = base + ((long)b * 32 + r) * 16;
    uint8_t* p1 = base + (long)nb * 512 + ((long)b * 32 + r) * 16;
    uint8_t* pd = base + (long)nb * 1024 + ((long)b * 32 + r) * 2;
    for (int i = 0; i < 16; ++i) { p0[i] = in[2 + i]; p1[i] = in[18 + i]; }
    pd[0] = in[0];
    pd[1] = in[1];
  }
}

}  // namespace fox
