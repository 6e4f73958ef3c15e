// Dequantise-GEMV kernels for batch-1 decode (sm_100a).
//
// One CTA owns one unit of U whole rows at a time (pack.cuh): thread t decodes
// block t % nb of row t / nb, so a thread's slice of the activation vector is
// the same for every unit and lives in registers for the whole kernel. Per
// block the thread forms upstream's integer partial sums with __dp4a, turns
// them into the float terms upstream forms, and parks them in shared memory;
// one thread per row then adds the row's terms in upstream's block order, so a
// row comes out bit-identical to upstream's CPU kernel given the same input.
//
//   TQ1_0/TQ2_0  per-vector int8 activations  upstream src/gemv.c:11-97,
//                src/ternary.c:59-93,177-188,226-246
//   Q4_K/Q6_K    per-256 int8 activations     upstream src/kernels.c:465-500,
//                531-569,571-602,636-661,722-805
//   Q8_0         float activations            upstream src/kernels.c:98-113
//
// Prologues fold upstream's per-call work into every CTA (each recomputes it
// from the L2-resident input vector, so no extra launch or grid sync):
//   PRO_PREQ    int8 activations and scale(s) given
//   PRO_VEC     float vector -> upstream's quantiser
//   PRO_NORM    residual -> RMSNorm (double sum of squares, src/ops.c:7-22) ->
//               upstream's quantiser
//   PRO_GSCALE  a tensor-parallel shard of a float vector, quantised with the
//               absmax of the whole vector (xq_scale[0], from all shards), so
//               its int8 values are the ones the unsplit vector gets
//   PRO_XAMAX   as PRO_GSCALE, with the whole vector's absmax traded over
//               peer memory inside the kernel (p2p.cuh slots): every CTA
//               publishes the shard's absmax to every rank and takes the
//               largest of all ranks' slots
//   PRO_NFOLD   as PRO_NORM, with the residual first completed from a
//               partial-sum exchange over peer memory: x = the ranks' row
//               sums added in rank order (rank 0's carries the residual),
//               each read from this rank's arena once it carries the
//               exchange's epoch; CTA 0 stores the completed residual back
// EPI_TERMS (tensor-parallel row shards) writes the per-block float terms
// instead of folding them; the shards' terms are gathered and folded in
// upstream's block order by fold_kernel (fold_x_kernel over peer memory,
// where the CTA that finishes last publishes this rank's readiness).
// EPI_XSUM (tensor-parallel row shards, partial-sum exchange) stores each
// row's value, this shard's blocks folded in order times the activation
// scale (rank 0 adds the residual), as an {epoch, value} word into this
// rank's slot of every rank's arena.
// Epilogues: store; residual add (src/ops.c:50-54); RoPE on adjacent pairs
// (src/ops.c:56-73) + K/V cache write for the fused q|k|v matrix; SwiGLU
// (src/ops.c:41-48) for the interleaved gate|up matrix.
#pragma once

#include "common.cuh"
#include "p2p.cuh"
#include "pack.cuh"

namespace fox {

enum Pro { PRO_PREQ = 0, PRO_VEC = 1, PRO_NORM = 2, PRO_GSCALE = 3, PRO_XAMAX = 4, PRO_NFOLD = 5 };
enum Epi { EPI_STORE = 0, EPI_ADD = 1, EPI_QKV = 2, EPI_SWIGLU = 3, EPI_TERMS = 4, EPI_XSUM = 5 };

// Largest CTA per type: 64 activation registers plus a prefetched unit must
// fit the register file at this width.
__host__ __device__ constexpr int gemv_max_threads(int t) {
  return (t == T_Q4_K || t == T_Q6_K) ? 256 : 512;
}
constexpr int XQ_STRIDE = 272;  // padded bytes per 256-block of int8 activations

struct GemvParams {
  const uint8_t* w;  // packed weights
  int n_rows, K, nb, U;
  const float* x;         // PRO_VEC / PRO_NORM input, K floats
  const float* norm_w;    // PRO_NORM weight, K floats
  float eps;
  const int8_t* xq;       // PRO_PREQ activations, K int8
  const float* xq_scale;  // PRO_PREQ scale(s): 1 (ternary) or K/256 (K-quants)
  float* out;             // STORE/ADD: n_rows; SWIGLU: n_rows/2; QKV: the q rows
  // EPI_QKV
  int nq, nkv, hd, n_ctx, kv_f16;
  const float* rope_cos;  // [n_ctx][hd/2]
  const float* rope_sin;
  const int* pos;
  void* kcache;           // this layer's caches (common.cuh kv_row)
  void* vcache;
  const int* kv_table;    // the block table of a paged cache (nullptr: contiguous)
  int row_base;           // first row of this matrix within q|k|v
  int* err;               // set to a nonzero code when a bounded device wait gives up
  // ring mode: units stream through ring_slots shared-memory slots of
  // slot_bytes each, starting ring_off bytes into dynamic shared memory
  int ring_slots, slot_bytes, ring_off;
  // EPI_TERMS: row r's block terms go to out[r * terms_stride + i]
  int terms_stride;
  // launch with programmatic stream serialisation (overlap the predecessor);
  // only where every predecessor in the stream is a kernel of this chain
  int pdl;
  // exchanges over peer memory (p2p.cuh), epochs from `pos`. PRO_XAMAX
  // publishes into slot [x_which][x_rank] of every arena, waits for all
  // ranks' slots in its own, and CTA 0 stores the result to x_amax (for the
  // fold). EPI_TERMS with x_count set: each CTA counts itself done there and
  // the last one publishes readiness [x_which][x_rank] in every arena.
  uint8_t* x_peers[TPX_MAX];
  int x_rank, x_world, x_which, x_phase;
  unsigned* x_count;
  float* x_amax;
  // EPI_XSUM: the partial-sum area of this projection (byte offset in every
  // arena, [rank][n_rows] floats) and the residual rank 0 adds
  size_t x_y_off;
  const float* x_res;
  // PRO_NFOLD: the partial-sum area to complete the residual from, its
  // readiness slot and epoch phase, and where CTA 0 stores the residual
  size_t f_y_off;
  int f_which, f_phase;
  float* f_out;
};

__host__ __device__ constexpr bool pro_norms(int pro) { return pro == PRO_NORM || pro == PRO_NFOLD; }

// PRO_NFOLD: elements i..i+3 of the residual completed from a sums exchange:
// the ranks' {epoch, value} words read until each carries this exchange's
// epoch (bounded; a wait that gives up sets the error word to 2 and *ok to
// false), the values added in rank order.
FOX_DEV float4 nfold_x4(const GemvParams& p, int i, int n, uint32_t ep, bool* ok) {
  const uint64_t* y = reinterpret_cast<const uint64_t*>(p.x_peers[p.x_rank] + p.f_y_off);
  float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int k = 0; k < p.x_world; ++k) {
    const uint64_t* w = y + (size_t)k * n + i;
    uint64_t v0 = 0, v1 = 0, v2 = 0, v3 = 0;
    bool got = false;
    for (int it = 0; it < (1 << 22); ++it) {
      ld_volatile_v2(w, v0, v1);
      ld_volatile_v2(w + 2, v2, v3);
      if ((uint32_t)(v0 >> 32) == ep && (uint32_t)(v1 >> 32) == ep && (uint32_t)(v2 >> 32) == ep &&
          (uint32_t)(v3 >> 32) == ep) {
        got = true;
        break;
      }
      if (it >= 16) __nanosleep(64);
      if ((it & 255) == 255 && step_failed(p.err)) break;
    }
    if (!got) {
      if (p.err) atomicExch(p.err, 2);
      *ok = false;
    }
    const float4 b = make_float4(__uint_as_float((uint32_t)v0), __uint_as_float((uint32_t)v1),
                                 __uint_as_float((uint32_t)v2), __uint_as_float((uint32_t)v3));
    if (k == 0) {
      a = b;
    } else {
      a.x = __fadd_rn(a.x, b.x); a.y = __fadd_rn(a.y, b.y);
      a.z = __fadd_rn(a.z, b.z); a.w = __fadd_rn(a.w, b.w);
    }
  }
  return a;
}

// EPI_XSUM: row r's value v as an {epoch, value} word into this rank's slot
// of every rank's arena (rank 0's carries the residual).
FOX_DEV void xsum_store(const GemvParams& p, int r, float v, uint32_t ep) {
  if (p.x_rank == 0) v = __fadd_rn(p.x_res[r], v);
  const uint64_t word = ((uint64_t)ep << 32) | __float_as_uint(v);
  for (int k = 0; k < p.x_world; ++k)
    st_relaxed_sys(reinterpret_cast<uint64_t*>(p.x_peers[k] + p.x_y_off) + (size_t)p.x_rank * p.n_rows + r, word);
}

// PRO_XAMAX: the largest absmax over all ranks. Every CTA publishes the same
// shard value, so no CTA waits on another CTA of its own grid; a wait that
// gives up sets the error word to 2 and yields 0 (the terms are then
// garbage, and the host reports the word).
FOX_DEV float x_trade_amax(const GemvParams& p, float am) {
  __shared__ float g_sh;
  if (threadIdx.x == 0) {
    const uint32_t ep = tp_epoch(p.pos, p.x_phase);
    const uint64_t word = ((uint64_t)ep << 32) | __float_as_uint(am);
    for (int k = 0; k < p.x_world; ++k)
      st_relaxed_sys(reinterpret_cast<uint64_t*>(p.x_peers[k] + AR_AMAX) + p.x_which * TPX_MAX + p.x_rank, word);
    const uint64_t* mine = reinterpret_cast<const uint64_t*>(p.x_peers[p.x_rank] + AR_AMAX) + p.x_which * TPX_MAX;
    float g = 0.0f;
    for (int k = 0; k < p.x_world; ++k) {
      uint64_t w = 0;
      if (!wait_hi(mine + k, ep, &w, p.err)) {
        if (p.err) atomicExch(p.err, 2);
        g = 0.0f;
        break;
      }
      g = fmaxf(g, __uint_as_float((uint32_t)w));
    }
    if (blockIdx.x == 0 && p.x_amax) *p.x_amax = g;
    g_sh = g;
  }
  __syncthreads();
  return g_sh;
}

// EPI_TERMS under the peer exchange: this CTA's terms are written; the CTA
// that counts itself last publishes this rank's readiness in every arena
// and rearms the counter for the next launch (stream-ordered after this
// one). Every thread fences its own terms at system scope before the count
// (the last-block pattern), so a peer that acquires the flag sees them all.
FOX_DEV void x_signal_ready(const GemvParams& p) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return;
  if (atomicAdd(p.x_count, 1u) != gridDim.x - 1) return;
  __threadfence_system();
  *p.x_count = 0u;
  const uint32_t ep = tp_epoch(p.pos, p.x_phase);
  for (int k = 0; k < p.x_world; ++k)
    st_release_sys(reinterpret_cast<uint32_t*>(p.x_peers[k] + AR_READY) + p.x_which * TPX_MAX + p.x_rank, ep);
}

// ---------------------------------------------------------------------------
// per-type block decoders

template <int T> struct W;

// TQ1_0: 5 base-3 levels per qs byte, 4 per qh byte. The level-l trit of byte
// c is ((c*3^l mod 256)*3) >> 8; two bytes per 32-bit register (16-bit lanes)
// are stepped together: p = q*3, trit = p >> 8 (a byte_perm collects the four
// trits of a word), q' = p & 0xFF. The -1 offset is folded in as -sum(x).
template <int L>
FOX_DEV int tq1_word(uint32_t c, const uint32_t* xw, int x0, int xs, int acc) {
  uint32_t lo = c & 0x00FF00FFu, hi = (c >> 8) & 0x00FF00FFu;
#pragma unroll
  for (int l = 0; l < L; ++l) {
    const uint32_t pl = lo * 3u, ph = hi * 3u;
    acc = dp4a(__byte_perm(pl, ph, 0x7351), xw[x0 + l * xs], acc);
    lo = pl & 0x00FF00FFu;
    hi = ph & 0x00FF00FFu;
  }
  return acc;
}

template <> struct W<T_TQ1_0> {
  static constexpr int NT = 1, BE = 256, MAXT = 512;
  static constexpr bool PREFETCH = true;
  struct R { uint4 a, b, c; uint32_t h, d; };
  template <bool SH = false>
  static FOX_DEV void load(R& r, const uint8_t* base, long cnt, int t) {
    r.a = ld16<SH>(base + t * 16);
    r.b = ld16<SH>(base + cnt * 16 + t * 16);
    r.c = ld16<SH>(base + cnt * 32 + t * 16);
    r.h = ld4<SH>(base + cnt * 48 + t * 4);
    r.d = ld2<SH>(base + cnt * 52 + t * 2);
  }
  // elements: l*32+m (qs[m], m<32), 160+l*16+m (qs[32+m]), 240+l*4+m (qh[m])
  static FOX_DEV int isum(const R& r, const uint32_t* xw, int sx) {
    const uint32_t c[12] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w,
                            r.c.x, r.c.y, r.c.z, r.c.w};
    int acc = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) acc = tq1_word<5>(c[w], xw, w, 8, acc);
#pragma unroll
    for (int w = 0; w < 4; ++w) acc = tq1_word<5>(c[8 + w], xw, 40 + w, 4, acc);
    acc = tq1_word<4>(r.h, xw, 60, 1, acc);
    return acc - sx;
  }
  static FOX_DEV void terms(const R& r, const uint32_t* xw, int sx, float, float* out) {
    out[0] = __fmul_rn(h2f((uint16_t)r.d), __int2float_rn(isum(r, xw, sx)));
  }
};

// TQ2_0: element j*128 + l*32 + m is bits 2l..2l+1 of qs[j*32+m], minus 1.
template <> struct W<T_TQ2_0> {
  static constexpr int NT = 1, BE = 256, MAXT = 512;
  static constexpr bool PREFETCH = true;
  struct R { uint4 q[4]; uint32_t d; };
  template <bool SH = false>
  static FOX_DEV void load(R& r, const uint8_t* base, long cnt, int t) {
#pragma unroll
    for (int i = 0; i < 4; ++i) r.q[i] = ld16<SH>(base + cnt * 16 * i + t * 16);
    r.d = ld2<SH>(base + cnt * 64 + t * 2);
  }
  static FOX_DEV int isum(const R& r, const uint32_t* xw, int sx) {
    const uint32_t c[16] = {r.q[0].x, r.q[0].y, r.q[0].z, r.q[0].w, r.q[1].x, r.q[1].y,
                            r.q[1].z, r.q[1].w, r.q[2].x, r.q[2].y, r.q[2].z, r.q[2].w,
                            r.q[3].x, r.q[3].y, r.q[3].z, r.q[3].w};
    // per level: mask in place (codes times 4^l), sum apart, shift back exactly
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int w = 0; w < 16; ++w)
#pragma unroll
      for (int l = 0; l < 4; ++l)
        acc[l] = dp4a_us(c[w] & (0x03030303u << (2 * l)), xw[(w >> 3) * 32 + l * 8 + (w & 7)], acc[l]);
    return acc[0] + (acc[1] >> 2) + (acc[2] >> 4) + (acc[3] >> 6) - sx;
  }
  static FOX_DEV void terms(const R& r, const uint32_t* xw, int sx, float, float* out) {
    out[0] = __fmul_rn(h2f((uint16_t)r.d), __int2float_rn(isum(r, xw, sx)));
  }
};

// Q4_K: sub-block j (32 elements) = nibble (low for even j, high for odd) of
// qs[(j/2)*32 + l]; 6-bit scale/min packed as upstream src/kernels.c:246-255.
// Term j = ascale * (d*sc*dot - dmin*m*sum(x)) (src/kernels.c:591-598).
template <> struct W<T_Q4_K> {
  static constexpr int NT = 8, BE = 256, MAXT = 256;
  static constexpr bool PREFETCH = false;
  struct R { uint4 q[8]; uint32_t s0, s1, s2, dm; };
  template <bool SH = false>
  static FOX_DEV void load(R& r, const uint8_t* base, long cnt, int t) {
#pragma unroll
    for (int i = 0; i < 8; ++i) r.q[i] = ld16<SH>(base + cnt * 16 * i + t * 16);
    r.s0 = ld4<SH>(base + cnt * 128 + t * 4);
    r.s1 = ld4<SH>(base + cnt * 132 + t * 4);
    r.s2 = ld4<SH>(base + cnt * 136 + t * 4);
    r.dm = ld4<SH>(base + cnt * 140 + t * 4);
  }
  static FOX_DEV void scale_min(const R& r, int j, int& sc, int& m) {
    const uint32_t sw[3] = {r.s0, r.s1, r.s2};
#define SB(i) ((int)((sw[(i) >> 2] >> (8 * ((i) & 3))) & 0xffu))
    if (j < 4) { sc = SB(j) & 63; m = SB(j + 4) & 63; }
    else { sc = (SB(j + 4) & 0x0F) | ((SB(j - 4) >> 6) << 4); m = (SB(j + 4) >> 4) | ((SB(j) >> 6) << 4); }
#undef SB
  }
  // integer dot of sub-block j's nibbles with x, and the sum of x
  static FOX_DEV void sub(const R& r, const uint32_t* xw, int j, int& dot, int& sum) {
    const uint4 a = r.q[(j >> 1) * 2], b = r.q[(j >> 1) * 2 + 1];
    const uint32_t words[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    dot = 0; sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      dot = dp4a((words[k] >> (4 * (j & 1))) & 0x0F0F0F0Fu, xw[j * 8 + k], dot);
      sum = dp4a(0x01010101u, xw[j * 8 + k], sum);
    }
  }
  static FOX_DEV void ipart(const R& r, const uint32_t* xw, int32_t* out) {
#pragma unroll
    for (int j = 0; j < 8; ++j) sub(r, xw, j, out[2 * j], out[2 * j + 1]);
  }
  static FOX_DEV void terms(const R& r, const uint32_t* xw, int, float as, float* out) {
    const float d = h2f((uint16_t)(r.dm & 0xffff)), dmin = h2f((uint16_t)(r.dm >> 16));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int sc, m, dot, sum;
      scale_min(r, j, sc, m);
      sub(r, xw, j, dot, sum);
      const float a = __fmul_rn(__fmul_rn(d, (float)sc), __int2float_rn(dot));
      const float b = __fmul_rn(__fmul_rn(dmin, (float)m), __int2float_rn(sum));
      out[j] = __fmul_rn(as, __fsub_rn(a, b));
    }
  }
};

// Q6_K: group (half, sub) = sum over k of int8 scale[half*8 + sub + 2k] times
// the dot of the signed 6-bit values of run k with x (src/kernels.c:531-569).
// Term = (ascale * d) * group (src/kernels.c:654-657).
template <> struct W<T_Q6_K> {
  static constexpr int NT = 4, BE = 256, MAXT = 256;
  static constexpr bool PREFETCH = false;
  struct R { uint4 ql[8]; uint4 qh[4]; uint4 sc; uint32_t d; };
  template <bool SH = false>
  static FOX_DEV void load(R& r, const uint8_t* base, long cnt, int t) {
#pragma unroll
    for (int i = 0; i < 8; ++i) r.ql[i] = ld16<SH>(base + cnt * 16 * i + t * 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) r.qh[i] = ld16<SH>(base + cnt * (128 + 16 * i) + t * 16);
    r.sc = ld16<SH>(base + cnt * 192 + t * 16);
    r.d = ld2<SH>(base + cnt * 208 + t * 2);
  }
  static FOX_DEV uint32_t wd(const uint4* v, int i) {
    return (i & 3) == 0 ? v[i >> 2].x : (i & 3) == 1 ? v[i >> 2].y : (i & 3) == 2 ? v[i >> 2].z : v[i >> 2].w;
  }
  static FOX_DEV int group(const R& r, const uint32_t* xw, int half, int sub) {
    const uint32_t scw[4] = {r.sc.x, r.sc.y, r.sc.z, r.sc.w};
    int g = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      int dot = 0, s = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t ql = wd(r.ql, half * 16 + (k & 1) * 8 + sub * 4 + i);
        const uint32_t qh = wd(r.qh, half * 8 + sub * 4 + i);
        const uint32_t q = ((ql >> (4 * (k >> 1))) & 0x0F0F0F0Fu) |
                           (((qh >> (2 * k)) & 0x03030303u) << 4);
        const uint32_t xv = xw[half * 32 + 8 * k + sub * 4 + i];
        dot = dp4a(q, xv, dot);
        s = dp4a(0x01010101u, xv, s);
      }
      const int si = half * 8 + sub + 2 * k;
      const int scale = (int)(int8_t)((scw[si >> 2] >> (8 * (si & 3))) & 0xffu);
      g += scale * (dot - 32 * s);
    }
    return g;
  }
  static FOX_DEV void ipart(const R& r, const uint32_t* xw, int32_t* out) {
#pragma unroll
    for (int g = 0; g < 4; ++g) out[g] = group(r, xw, g >> 1, g & 1);
  }
  static FOX_DEV void terms(const R& r, const uint32_t* xw, int, float as, float* out) {
    const float ad = __fmul_rn(as, h2f((uint16_t)r.d));
#pragma unroll
    for (int g = 0; g < 4; ++g) out[g] = __fmul_rn(ad, __int2float_rn(group(r, xw, g >> 1, g & 1)));
  }
};

// Q8_0 against float activations: acc over the 32 elements in order, then
// d * acc (src/kernels.c:98-113). int8 -> float via byte_perm into the
// mantissa of 2^23 and one exact subtraction.
template <> struct W<T_Q8_0> {
  static constexpr int NT = 1, BE = 32, MAXT = 512;
  static constexpr bool PREFETCH = true;
  struct R { uint4 a, b; uint32_t d; };
  template <bool SH = false>
  static FOX_DEV void load(R& r, const uint8_t* base, long cnt, int t) {
    r.a = ld16<SH>(base + t * 16);
    r.b = ld16<SH>(base + cnt * 16 + t * 16);
    r.d = ld2<SH>(base + cnt * 32 + t * 2);
  }
  static FOX_DEV void termsf(const R& r, const float* xf, float* out) {
    const uint32_t c[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
    float acc = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t v = c[w] ^ 0x80808080u;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float q = __fsub_rn(__uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540 + k)), 8388736.0f);
        acc = __fadd_rn(acc, __fmul_rn(q, xf[4 * w + k]));
      }
    }
    out[0] = __fmul_rn(h2f((uint16_t)r.d), acc);
  }
};

template <int T> constexpr bool is_ternary() { return T == T_TQ1_0 || T == T_TQ2_0; }
template <int T> constexpr bool is_kquant() { return T == T_Q4_K || T == T_Q6_K; }

// Shared memory bytes a launch needs.
inline size_t gemv_smem_bytes(int type, int pro, int K, int U, int nb) {
  size_t s = 0;
  if (pro != PRO_PREQ) s += (size_t)(K + K / 8) * 4;              // staged (padded) floats
  if (type != T_Q8_0) s += (size_t)(K / 256) * XQ_STRIDE + (K / 256) * 4;  // int8 + scales
  s = (s + 15) / 16 * 16;
  s += 32 * 8;                                                    // reduction scratch
  const int nt = type == T_Q4_K ? 8 : type == T_Q6_K ? 4 : 1;
  s += (size_t)U * (nb * nt + 1) * 4 + (size_t)U * 4;
  return s;
}

// ---------------------------------------------------------------------------

// RING: instead of a register prefetch of the next unit, thread 0 keeps up to
// ring_slots of this CTA's units in flight as bulk asynchronous copies into
// shared memory (one mbarrier per slot, reissued as soon as a slot has been
// read), so a CTA has tens of KB of weights in flight instead of one unit.
// A ring launch carries programmatic stream serialisation: the first copies
// start before the predecessor kernel has finished.
template <int T, int PRO, int EPI, bool RING = false>
__global__ void __launch_bounds__(W<T>::MAXT)
gemv_kernel(const GemvParams p) {
  using Tr = W<T>;
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, nth = blockDim.x;
  const int K = p.K, nb = p.nb, U = p.U, ut = U * nb;
  const int nb256 = K / 256;
  const int units = (p.n_rows + U - 1) / U;
  const long unit_bytes = (long)ut * block_bytes(T);

  uint8_t* ring = smem + p.ring_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + (size_t)p.ring_slots * p.slot_bytes);
  const int R = p.ring_slots;
  const int n_mine = (int)blockIdx.x < units ? (units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  // A partial last unit whose size is not a multiple of 16 bytes cannot be
  // bulk-copied; it is read from global memory directly (it is always the
  // last unit of its CTA, so no later use of its slot is affected).
  auto direct = [&](int u) {
    const int ru = min(U, p.n_rows - u * U);
    return ((long)ru * nb * block_bytes(T)) % 16 != 0;
  };
  // the k-th unit of this CTA into slot k % R
  auto issue = [&](int k) {
    const int uu = blockIdx.x + k * gridDim.x;
    if (direct(uu)) return;
    const int ru = min(U, p.n_rows - uu * U);
    const unsigned bytes = (unsigned)((long)ru * nb * block_bytes(T));
    uint64_t* b = bars + k % R;
    mbar_arrive_expect_tx(b, bytes);
    bulk_g2s(ring + (size_t)(k % R) * p.slot_bytes, p.w + (size_t)uu * unit_bytes, bytes, b);
  };
  if (RING) {
    if (tid == 0) {
      for (int i = 0; i < R; ++i) mbar_init(bars + i, 1);
      mbar_fence_init();
      for (int k = 0; k < min(R, n_mine); ++k) issue(k);
    }
    griddep_launch_dependents();
    griddep_wait();
    __syncthreads();
  }

  unsigned char* sp = smem;
  float* xs = nullptr;
  if (PRO != PRO_PREQ) { xs = (float*)sp; sp += (size_t)(K + K / 8) * 4; }
  int8_t* xq = nullptr;
  float* ascale = nullptr;
  if (T != T_Q8_0) {
    xq = (int8_t*)sp; sp += (size_t)nb256 * XQ_STRIDE;
    ascale = (float*)sp; sp += nb256 * 4;
  }
  sp = (unsigned char*)(((uintptr_t)sp + 15) & ~(uintptr_t)15);
  double* red = (double*)sp; sp += 32 * 8;
  // per-row term slots, row stride padded by one so the chain threads of a
  // unit read different banks
  const int rstride = nb * Tr::NT + 1;
  float* part = (float*)sp; sp += (size_t)U * rstride * 4;
  float* vals = (float*)sp;

  // Q8_0 keeps floats padded by 4 every 32 so per-thread 32-float reads of
  // different blocks fall in different banks.
  auto xsi = [&](int i) { return T == T_Q8_0 ? i + (i >> 5) * 4 : i; };

  // ---------------- prologue: the activation vector ----------------------
  if (PRO != PRO_PREQ) {
    const uint32_t fep = PRO == PRO_NFOLD ? tp_epoch(p.pos, p.f_phase) : 0u;
    bool fok = true;
    double ss = 0.0;
    for (int i = tid * 4; i < K; i += nth * 4) {
      const float4 v = PRO == PRO_NFOLD ? nfold_x4(p, i, K, fep, &fok) : *reinterpret_cast<const float4*>(p.x + i);
      if (PRO == PRO_NFOLD && blockIdx.x == 0) *reinterpret_cast<float4*>(p.f_out + i) = v;
      if (pro_norms(PRO))
        ss = ss + (double)v.x * (double)v.x + (double)v.y * (double)v.y +
             (double)v.z * (double)v.z + (double)v.w * (double)v.w;
      *reinterpret_cast<float4*>(xs + xsi(i)) = v;
    }
    if (pro_norms(PRO)) {
      const double sum = block_reduce<double>(ss, red, OpAddD(), 0.0);
      const float scale = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)K), (double)p.eps)));
      for (int i = tid * 4; i < K; i += nth * 4) {
        float4 v = *reinterpret_cast<float4*>(xs + xsi(i));
        const float4 w = *reinterpret_cast<const float4*>(p.norm_w + i);
        v.x = __fmul_rn(__fmul_rn(v.x, scale), w.x);
        v.y = __fmul_rn(__fmul_rn(v.y, scale), w.y);
        v.z = __fmul_rn(__fmul_rn(v.z, scale), w.z);
        v.w = __fmul_rn(__fmul_rn(v.w, scale), w.w);
        *reinterpret_cast<float4*>(xs + xsi(i)) = v;
      }
    }
    __syncthreads();
  }

  float act_scale = 1.0f;
  if (is_ternary<T>()) {
    if (PRO == PRO_PREQ) {
      act_scale = p.xq_scale[0];
    } else {
      // upstream src/gemv.c:11-42: one absmax over the whole vector
      float amax;
      if (PRO == PRO_GSCALE) {
        amax = p.xq_scale[0];
      } else {
        float am = 0.0f;
        for (int i = tid; i < K; i += nth) am = absmax_acc(am, xs[i]);
        amax = block_reduce<float>(am, (float*)red, OpMax(), 0.0f);
        if (PRO == PRO_XAMAX) amax = x_trade_amax(p, amax);
      }
      const bool nz = amax > 0.0f;
      const float inv = nz ? __fdiv_rn(127.0f, amax) : 0.0f;
      act_scale = nz ? __fdiv_rn(amax, 127.0f) : 0.0f;
      for (int i = tid * 4; i < K; i += nth * 4) {
        const float4 v = *reinterpret_cast<const float4*>(xs + i);
        *reinterpret_cast<uint32_t*>(xq + (i >> 8) * XQ_STRIDE + (i & 255)) =
            pack4(quant1(v.x, inv), quant1(v.y, inv), quant1(v.z, inv), quant1(v.w, inv));
      }
    }
  } else if (is_kquant<T>()) {
    if (PRO == PRO_PREQ) {
      for (int b = tid; b < nb256; b += nth) ascale[b] = p.xq_scale[b];
    } else {
      // upstream src/kernels.c:722-754: one absmax per 256 block, a warp each
      const int lane = tid & 31, warp = tid >> 5, nw = nth >> 5;
      for (int b = warp; b < nb256; b += nw) {
        float v[8], am = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) { v[k] = xs[b * 256 + lane * 8 + k]; am = absmax_acc(am, v[k]); }
        am = warp_max(am);
        const bool nz = am > 0.0f;
        const float inv = nz ? __fdiv_rn(127.0f, am) : 0.0f;
        uint32_t* dst = reinterpret_cast<uint32_t*>(xq + b * XQ_STRIDE + lane * 8);
        dst[0] = pack4(quant1(v[0], inv), quant1(v[1], inv), quant1(v[2], inv), quant1(v[3], inv));
        dst[1] = pack4(quant1(v[4], inv), quant1(v[5], inv), quant1(v[6], inv), quant1(v[7], inv));
        if (lane == 0) ascale[b] = nz ? __fdiv_rn(am, 127.0f) : 0.0f;
      }
    }
  }
  if (PRO != PRO_PREQ || is_kquant<T>()) __syncthreads();

  // per-thread activation slice
  const int blk = tid < ut ? tid % nb : 0;
  uint32_t xw[T == T_Q8_0 ? 1 : 64];
  float xf[T == T_Q8_0 ? 32 : 1];
  int sx = 0;
  float as = 1.0f;
  if (T == T_Q8_0) {
#pragma unroll
    for (int k = 0; k < 32; k += 4) {
      const float4 v = *reinterpret_cast<const float4*>(xs + xsi(blk * 32 + k));
      xf[k] = v.x; xf[k + 1] = v.y; xf[k + 2] = v.z; xf[k + 3] = v.w;
    }
  } else {
    if (PRO == PRO_PREQ) {
      const uint4* src = reinterpret_cast<const uint4*>(p.xq + (size_t)blk * 256);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint4 v = src[i];
        xw[4 * i] = v.x; xw[4 * i + 1] = v.y; xw[4 * i + 2] = v.z; xw[4 * i + 3] = v.w;
      }
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(xq + blk * XQ_STRIDE);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint4 v = src[i];
        xw[4 * i] = v.x; xw[4 * i + 1] = v.y; xw[4 * i + 2] = v.z; xw[4 * i + 3] = v.w;
      }
    }
#pragma unroll
    for (int i = 0; i < 64; ++i) sx = dp4a(0x01010101u, xw[i], sx);
    if (is_kquant<T>()) as = ascale[blk];
  }

  // ---------------- main loop over units ---------------------------------
  const int prow = tid / nb, pcol = (tid - prow * nb) * Tr::NT;
  // rows of unit u in upstream's order from the parked terms, then the epilogue
  auto finish = [&](int u, int ru) {
    if (EPI == EPI_TERMS) {
      const int tr = nb * Tr::NT;
      for (int i = tid; i < ru * tr; i += nth) {
        const int r = i / tr, c = i - r * tr;
        p.out[(size_t)(u * U + r) * p.terms_stride + c] = part[r * rstride + c];
      }
      __syncthreads();
      return;
    }
    float v = 0.0f;
    if (tid < ru) {
      // upstream order: blocks in order, terms of a block in order, from 0.0f
      const float* pr = part + tid * rstride;
      float acc = 0.0f;
      for (int i = 0; i < nb * Tr::NT; ++i) acc = __fadd_rn(acc, pr[i]);
      v = is_ternary<T>() ? __fmul_rn(acc, act_scale) : acc;
      const int r = u * U + tid;
      if (EPI == EPI_STORE) p.out[r] = v;
      if (EPI == EPI_ADD) p.out[r] = __fadd_rn(p.out[r], v);
      if (EPI == EPI_XSUM) xsum_store(p, r, v, tp_epoch(p.pos, p.x_phase));
      if (EPI == EPI_QKV || EPI == EPI_SWIGLU) vals[tid] = v;
    }
    if (EPI == EPI_QKV || EPI == EPI_SWIGLU) {
      __syncthreads();
      if (EPI == EPI_QKV && tid < ru) {
        const int r = p.row_base + u * U + tid;
        const int P = *p.pos;
        const float mine = vals[tid];
        if (r < p.nq + p.nkv) {
          const float other = vals[tid ^ 1];
          const int rr = r < p.nq ? r : r - p.nq;
          const int i = (rr % p.hd) >> 1;
          const float c = p.rope_cos[(size_t)P * (p.hd >> 1) + i];
          const float s = p.rope_sin[(size_t)P * (p.hd >> 1) + i];
          const bool odd = tid & 1;
          const float x0 = odd ? other : mine, x1 = odd ? mine : other;
          const float o = odd ? __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c))
                              : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
          if (r < p.nq) {
            p.out[r] = o;
          } else {
            const size_t idx = kv_row(p.kv_table, p.n_ctx, p.nkv / p.hd, rr / p.hd, P) * p.hd + rr % p.hd;
            if (p.kv_f16) reinterpret_cast<__half*>(p.kcache)[idx] = __float2half_rn(o);
            else reinterpret_cast<float*>(p.kcache)[idx] = o;
          }
        } else {
          const int rr = r - p.nq - p.nkv;
          const size_t idx = kv_row(p.kv_table, p.n_ctx, p.nkv / p.hd, rr / p.hd, P) * p.hd + rr % p.hd;
          if (p.kv_f16) reinterpret_cast<__half*>(p.vcache)[idx] = __float2half_rn(mine);
          else reinterpret_cast<float*>(p.vcache)[idx] = mine;
        }
      }
      if (EPI == EPI_SWIGLU && tid < (ru >> 1)) {
        const float g = vals[tid], up = vals[tid + (ru >> 1)];
        p.out[u * (U >> 1) + tid] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf_up(-g))), up);
      }
    }
    __syncthreads();
  };
  auto park = [&](const typename Tr::R& w) {
    float t[Tr::NT];
    if constexpr (T == T_Q8_0) Tr::termsf(w, xf, t);
    else Tr::terms(w, xw, sx, as, t);
#pragma unroll
    for (int k = 0; k < Tr::NT; ++k) part[prow * rstride + pcol + k] = t[k];
  };

  typename Tr::R cur, nxt;
  if constexpr (RING) {
    for (int k = 0; k < n_mine; ++k) {
      const int u = blockIdx.x + k * gridDim.x;
      const int ru = min(U, p.n_rows - u * U);
      const int slot = k % R;
      const bool dir = direct(u);
      const bool got = dir || mbar_wait(bars + slot, (k / R) & 1);
      if (!__syncthreads_and(got)) {
        if (tid == 0) {
          if (p.err) atomicExch(p.err, 2);
          // a second bounded wait for every copy still in flight
          for (int j = k; j < min(n_mine, k + R); ++j)
            if (!direct(blockIdx.x + j * gridDim.x)) mbar_wait(bars + j % R, (j / R) & 1);
        }
        __syncthreads();
        // still counted, so the completion count is rearmed for the next
        // exchange; the error word marks this step's terms as unusable
        if (EPI == EPI_TERMS && p.x_count) x_signal_ready(p);
        return;
      }
      if (tid < ru * nb) {
        if (dir) Tr::load(cur, p.w + u * unit_bytes, (long)ru * nb, tid);
        else Tr::template load<true>(cur, ring + (size_t)slot * p.slot_bytes, (long)ru * nb, tid);
        park(cur);
      }
      __syncthreads();  // the slot is free again
      if (tid == 0 && k + R < n_mine) issue(k + R);
      finish(u, ru);
    }
  } else {
    int u = blockIdx.x;
    if (Tr::PREFETCH && u < units) {
      const int ru = min(U, p.n_rows - u * U);
      if (tid < ru * nb) Tr::load(cur, p.w + u * unit_bytes, (long)ru * nb, tid);
    }
    for (; u < units; u += gridDim.x) {
      const int ru = min(U, p.n_rows - u * U);
      if (Tr::PREFETCH) {
        const int un = u + gridDim.x;
        if (un < units) {
          const int run = min(U, p.n_rows - un * U);
          if (tid < run * nb) Tr::load(nxt, p.w + un * unit_bytes, (long)run * nb, tid);
        }
      } else if (tid < ru * nb) {
        Tr::load(cur, p.w + u * unit_bytes, (long)ru * nb, tid);
      }
      if (tid < ru * nb) park(cur);
      __syncthreads();
      finish(u, ru);
      if (Tr::PREFETCH) cur = nxt;
    }
  }
  if (EPI == EPI_TERMS && p.x_count) x_signal_ready(p);
}

}  // namespace fox
