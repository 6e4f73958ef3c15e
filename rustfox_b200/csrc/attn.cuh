// Decode attention in tiles (sm_100a): the production form of upstream's
// attention_heads (src/forward.c:222-257, src/ops.c:24-39,75-81).
//
// The positions 0..P-1 are cut into tiles of T = ceil(P / NT) positions for
// the model's tile target NT (at most 8), so there are at most NT tiles. Per
// KV head g and tile t, one CTA forms for each query head of the group:
//   s_j = dot(q, k_j) * scale, the dot as 32 lane partials over hd/32 dims
//         each (q0*k0, then fmaf in dimension order) summed by an xor
//         butterfly (16, 8, 4, 2, 1);
//   m_t = max_j s_j;  e_j = expf(s_j - m_t);
//   l_t = sum_j e_j (ascending j);
//   o_t = sum_j fmaf(e_j, v_j, .) (ascending j, from 0).
// The NT CTAs of a KV head form one thread-block cluster; the tiles are
// merged through distributed shared memory, each CTA taking a share of the
// outputs:
//   M = max_t m_t;  w_t = expf(m_t - M);
//   L = sum_t fmaf(l_t, w_t, .);  O = sum_t fmaf(o_t, w_t, .)
//   (ascending t, from 0);  out = O / L.
// The oracle restates this order (or_ctx with a tile target, or_tile_attention).
//
// attention_exact_kernel (ops.cuh) keeps upstream's serial order (the parity
// mode).
#pragma once

#include <math_constants.h>

#include "ops.cuh"

namespace fox {

// Timestamps for an instrumented build (defined empty here).
#ifndef FOX_ATTN_MARK
#define FOX_ATTN_MARK(k)
#endif

constexpr int ATTN_TILE_MAX = 8;     // tile target NT: the tiles of a KV head form one portable cluster
constexpr int ATTN_TILE_GQA = 8;     // query heads per KV head

// Tile length for P positions and tile target nt.
__host__ __device__ inline int attn_tile_len(int P, int nt) { return (P + nt - 1) / nt; }

FOX_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
FOX_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

FOX_DEV unsigned cluster_ctarank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster; orders shared-memory writes
// before the barrier with reads after it, across the cluster.
FOX_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The same shared-memory variable in CTA `rank` of this cluster.
FOX_DEV const float* cluster_peer(const float* p, unsigned rank) {
  uint64_t r;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(p), "r"(rank));
  return reinterpret_cast<const float*>(r);
}

constexpr int ATTN_THREADS = 256;  // threads of a tile CTA (8 warps)
constexpr int ATTN_RING_MIN = 3;   // ring slots per CTA (nslot - 1 chunks in flight while one is read)
constexpr int ATTN_RING_MAX = 4;

// Every commit group but the newest nslot - 1 has landed (this thread's copies).
FOX_DEV void cp_async_wait_ring(int nslot) {
  if (nslot >= 4) asm volatile("cp.async.wait_group 3;" ::: "memory");
  else asm volatile("cp.async.wait_group 2;" ::: "memory");
}

// Where KV head g's positions of one sequence and layer live: the cache
// base, and its block table when paged (common.cuh kv_row).
struct KvHead {
  const uint8_t* base;
  const int* table;
  int n_ctx, n_kv, g, rb;  // rb: row bytes
  FOX_DEV const uint8_t* row(int pos) const { return base + kv_row(table, n_ctx, n_kv, g, pos) * rb; }
};

// Positions [r0, r1) of a head into buf, position r at (r - r0) * rb,
// except position `skip`; asynchronous (cp.async, L2 only), no commit. The
// row is rb / 16 pieces of 16 bytes and that count divides ATTN_THREADS
// (head_dim 64, 128 or 256), so each thread copies the same piece of every
// (ATTN_THREADS / pieces)-th row.
FOX_DEV void stage_rows(uint8_t* buf, const KvHead& kv, int r0, int r1, int skip) {
  const int per_row = kv.rb >> 4;
  const int col = (int)threadIdx.x % per_row, rstep = ATTN_THREADS / per_row;
  for (int row = (int)threadIdx.x / per_row; r0 + row < r1; row += rstep) {
    if (r0 + row == skip) continue;
    cp_async16(buf + (uint32_t)row * kv.rb + col * 16, kv.row(r0 + row) + col * 16);
  }
}

// NW consecutive 32-bit words from p (aligned to 4 * NW bytes, at most 16),
// with vector loads.
template <int NW>
FOX_DEV void load_words(const uint8_t* p, unsigned (&w)[NW]) {
  if constexpr (NW == 1) {
    w[0] = *reinterpret_cast<const unsigned*>(p);
  } else if constexpr (NW == 2) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    w[0] = u.x; w[1] = u.y;
  } else {
#pragma unroll
    for (int i = 0; i < NW / 4; ++i) {
      const uint4 u = reinterpret_cast<const uint4*>(p)[i];
      w[4 * i] = u.x; w[4 * i + 1] = u.y; w[4 * i + 2] = u.z; w[4 * i + 3] = u.w;
    }
  }
}

// Row r of a staged chunk as floats: DPL elements from element e0.
template <int DPL, bool F16>
FOX_DEV void staged_row(const uint8_t* buf, int r, int hd, int e0, float* v) {
  constexpr int ES = F16 ? 2 : 4, NW = DPL * ES / 4;
  unsigned w[NW];
  load_words<NW>(buf + ((uint32_t)r * hd + e0) * ES, w);
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    if (F16) {
      v[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xffffu)));
      v[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
    } else {
      v[i] = __uint_as_float(w[i]);
    }
  }
}

// Element d of row r of a staged chunk.
template <bool F16>
FOX_DEV float staged_one(const uint8_t* buf, int r, int hd, int d) {
  if (F16) return __half2float(reinterpret_cast<const __half*>(buf)[(uint32_t)r * hd + d]);
  return reinterpret_cast<const float*>(buf)[(uint32_t)r * hd + d];
}

// Scores of 8 rows held in registers (kf, the lane's hd/32 dimensions of
// each; at most `valid` rows) for one query head: lane l forms the partial
// over its dimensions for each row (q0*k0, then fmaf in dimension order),
// then a butterfly reduce-scatter (offsets 16, 8, 4) and two exchanges (2,
// 1) leave row (lane >> 2)'s dot in lanes 4k..4k+3. Every add pairs the
// same lane partials as an xor all-reduce (16, 8, 4, 2, 1) does, so each dot
// is the all-reduce's value bit for bit, with 9 exchanges for 8 rows
// instead of 40.
template <int DPL>
FOX_DEV float dot8(const float (&kf)[8][DPL], int valid, const float* qh, int lane) {
  float q[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) q[e] = qh[lane * DPL + e];
  float P[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    P[i] = 0.0f;
    if (i < valid) {
      float d = __fmul_rn(q[0], kf[i][0]);
#pragma unroll
      for (int e = 1; e < DPL; ++e) d = __fmaf_rn(q[e], kf[i][e], d);
      P[i] = d;
    }
  }
#pragma unroll
  for (int lv = 0; lv < 3; ++lv) {
    const int o = 16 >> lv, m = 8 >> lv;
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < m / 2; ++i) {
      const float send = up ? P[i] : P[i + m / 2];
      const float keep = up ? P[i + m / 2] : P[i];
      P[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
    }
  }
  const float r = __fadd_rn(P[0], __shfl_xor_sync(0xffffffffu, P[0], 2));
  return __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 1));
}

// Shared memory of a tile CTA (floats unless noted):
//   sc    G * ts     scores, then weights (ts: tile length rounded up to 4)
//   q     G * hd     the group's query heads
//   ml    64         per-head max [0, 32), sum [32, 64)
//   part  G * hd     this tile's unnormalised outputs (read by the cluster)
//   ring  nslot * ch * row bytes: staged chunks of K, then of V
struct TileSmem {
  float* sc;
  float* q;
  float* ml;
  float* part;
  uint8_t* ring;
  int ch, ts, slot, nslot;  // rows per chunk, score row stride, bytes per ring slot, slots
};

__host__ __device__ inline int attn_score_stride(int n_ctx, int nt) { return (attn_tile_len(n_ctx, nt) + 3) & ~3; }

inline size_t attn_tile_smem_bytes(int n_ctx, int nt, int gqa, int hd, int kv_f16, int ch, int nslot) {
  const size_t floats = (size_t)gqa * attn_score_stride(n_ctx, nt) + 2 * (size_t)gqa * hd + 64;
  return floats * 4 + (size_t)nslot * ch * hd * (kv_f16 ? 2 : 4);
}

FOX_DEV TileSmem tile_smem(float* base, int n_ctx, int nt, int gqa, int hd, int kv_f16, int ch, int nslot) {
  TileSmem m;
  m.ts = attn_score_stride(n_ctx, nt);
  m.sc = base;
  m.q = base + gqa * m.ts;
  m.ml = m.q + gqa * hd;
  m.part = m.ml + 64;
  m.ring = reinterpret_cast<uint8_t*>(m.part + gqa * hd);
  m.ch = ch;
  m.slot = ch * hd * (kv_f16 ? 2 : 4);
  m.nslot = nslot;
  return m;
}

struct TileArgs {
  const float* q;     // the group's query heads start at q + g * gqa * hd
  const void* kc;     // this layer's (and sequence's) caches (common.cuh kv_row)
  const void* vc;
  const int* table;   // block table of a paged cache (nullptr: contiguous)
  float* out;         // [n_head * hd]
  int n_ctx, n_kv, hd, nt, P;
  float scale;
  FOX_DEV KvHead head(const void* c, int g, int rb) const {
    return KvHead{reinterpret_cast<const uint8_t*>(c), table, n_ctx, n_kv, g, rb};
  }
};

// Tile t's positions [j0, j0 + n), nk chunks of ch rows.
struct TileGeom {
  int j0, n, nk;
};
FOX_DEV TileGeom tile_geom(const TileArgs& a, int t, int ch) {
  const int T = attn_tile_len(a.P, a.nt);
  TileGeom tg;
  tg.j0 = t * T;
  tg.n = min(T, a.P - tg.j0);
  tg.nk = (tg.n + ch - 1) / ch;
  return tg;
}

// Chunk c of the tile's staging order (K chunks 0..nk-1, then V chunks
// 0..nk-1) into ring slot c % nslot, without position `skip`; one commit
// group per call, empty past the last chunk.
FOX_DEV void attn_issue(const TileSmem& m, const KvHead& kh, const KvHead& vh, const TileGeom& tg, int c,
                        int skip) {
  if (c < 2 * tg.nk) {
    const bool isv = c >= tg.nk;
    const int r0 = tg.j0 + (isv ? c - tg.nk : c) * m.ch;
    KvHead src = kh;  // (a select of the base alone keeps both heads in registers)
    if (isv) src.base = vh.base;
    stage_rows(m.ring + (uint32_t)(c % m.nslot) * m.slot, src, r0, min(tg.j0 + tg.n, r0 + m.ch), skip);
  }
  cp_async_commit();
}

// The first nslot - 1 chunks of tile t of group g, without the newest
// position P - 1: everything they hold that earlier steps wrote, so they may
// be issued before griddepcontrol.wait.
template <bool F16>
FOX_DEV void attn_tile_stage0(const TileArgs& a, const TileSmem& m, int g, int t) {
  const int rb = a.hd * (F16 ? 2 : 4);
  const KvHead kh = a.head(a.kc, g, rb), vh = a.head(a.vc, g, rb);
  const TileGeom tg = tile_geom(a, t, m.ch);
  for (int c = 0; c < m.nslot - 1; ++c) attn_issue(m, kh, vh, tg, c, a.P - 1);
}

// Tile t of KV group g (after attn_tile_stage0): every query head's max,
// sum and unnormalised output into the CTA's shared memory (ml, part).
// The chunks stream through the ring, nslot - 1 in flight: the K chunks
// give the scores; after the last of them come the tile's max and the
// weights (while the first V chunks are in flight); the V chunks give the
// outputs and, in the same ascending order, the sums.
template <int DPL, bool F16, int G>
FOX_DEV void attn_tile(const TileArgs& a, const TileSmem& m, int g, int t) {
  constexpr int NW = ATTN_THREADS / 32;
  __shared__ float s_wm[NW];  // the max pass: each warp's max of its head
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hd = a.hd, ch = m.ch, ts = m.ts;
  const int rb = hd * (F16 ? 2 : 4);
  const KvHead kh = a.head(a.kc, g, rb), vh = a.head(a.vc, g, rb);
  const TileGeom tg = tile_geom(a, t, ch);
  const int j0 = tg.j0, n = tg.n, nk = tg.nk;
  const int newest = a.P - 1;
  float* sc = m.sc;
  float* s_m = m.ml;        // [G]
  float* s_l = m.ml + 32;   // [G]
  FOX_ATTN_MARK(1);
  for (int i = tid; i < G * hd; i += ATTN_THREADS) m.q[i] = __ldcg(a.q + (uint32_t)g * G * hd + i);
  // V chunks: thread (d, hg) sums dim d of heads hg, hg + hgs, ... (hpt of
  // them), each over the positions in order; the warps holding d < 32 also
  // sum the weights (thread d == 0 keeps them)
  const int hgs = max(1, min(G, ATTN_THREADS / hd)), hpt = G / hgs;
  const int d = tid % hd, hg = tid / hd;
  const bool vact = hg < hgs;
  const bool lsum = d < 32;  // uniform within a warp (hd is a multiple of 32)
  float o[G], l[G];
#pragma unroll
  for (int k = 0; k < G; ++k) o[k] = l[k] = 0.0f;
  for (int c = 0; c < 2 * nk; ++c) {
    attn_issue(m, kh, vh, tg, c + m.nslot - 1, -1);
    cp_async_wait_ring(m.nslot);  // chunk c has landed (this thread's copies)
    const bool isv = c >= nk;
    const int ci = isv ? c - nk : c;
    const int c0 = j0 + ci * ch, cn = min(ch, j0 + n - c0);
    const uint8_t* slot = m.ring + (uint32_t)(c % m.nslot) * m.slot;
    if (c < m.nslot - 1 && newest >= c0 && newest < c0 + cn) {
      // staged before the newest row was written: that row now
      KvHead h = kh;
      if (isv) h.base = vh.base;
      const unsigned* src = reinterpret_cast<const unsigned*>(h.row(newest));
      unsigned* dst = reinterpret_cast<unsigned*>(m.ring + (uint32_t)(c % m.nslot) * m.slot +
                                                  (uint32_t)(newest - c0) * rb);
      for (int i = tid; i < (rb >> 2); i += ATTN_THREADS) dst[i] = __ldcg(src + i);
    }
    __syncthreads();
    FOX_ATTN_MARK(2);
    if (!isv) {
      // tasks (group of 8 rows, head part): hsplit warps share a group,
      // the task of part p taking heads p, p + hsplit, ...; the rows stay in
      // registers across its heads
      const int groups = (cn + 7) >> 3;
      const int hsplit = min(G, NW / groups >= 8 ? 8 : NW / groups >= 4 ? 4 : NW / groups >= 2 ? 2 : 1);
      const int hpw = G / hsplit;
      for (int task = warp; task < groups * hsplit; task += NW) {
        const int r0 = (task / hsplit) * 8, hp = task % hsplit, valid = min(8, cn - r0);
        float kf[8][DPL];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i < valid) staged_row<DPL, F16>(slot, r0 + i, hd, lane * DPL, kf[i]);
#pragma unroll
        for (int k = 0; k < G; ++k) {
          if (k < hpw) {
            const int h = hp + k * hsplit;
            const float d = dot8<DPL>(kf, valid, m.q + h * hd, lane);
            const int r = r0 + (lane >> 2);
            if (!(lane & 3) && r < cn) sc[h * ts + ci * ch + r] = __fmul_rn(d, a.scale);
          }
        }
      }
      if (c == nk - 1) {
        // the tile's max per head (NW / G warps per head), then the weights
        __syncthreads();
        FOX_ATTN_MARK(3);
        constexpr int WPH = NW / G > 0 ? NW / G : 1;  // warps per head
        for (int h0 = 0; h0 < G; h0 += NW / WPH) {
          const int h = h0 + warp / WPH;
          float mx = -CUDART_INF_F;
          if (h < G)
            for (int j = (warp % WPH) * 32 + lane; j < n; j += WPH * 32) mx = fmaxf(mx, sc[h * ts + j]);
          mx = warp_max(mx);
          if (lane == 0) s_wm[warp] = mx;
          __syncthreads();
          if (tid < NW / WPH && h0 + tid < G) {
            float M = -CUDART_INF_F;
            for (int w = 0; w < WPH; ++w) M = fmaxf(M, s_wm[tid * WPH + w]);
            s_m[h0 + tid] = M;
          }
          __syncthreads();
        }
        for (int h = 0; h < G; ++h)
          for (int j = tid; j < n; j += ATTN_THREADS)
            sc[h * ts + j] = expf_up(__fsub_rn(sc[h * ts + j], s_m[h]));
        FOX_ATTN_MARK(4);
      }
    } else if (vact) {
      // the weights of 4 positions per shared-memory load
      const float* e = sc + ci * ch;
      int j = 0;
      for (; j + 4 <= cn; j += 4) {
        float4 w[G];
#pragma unroll
        for (int k = 0; k < G; ++k)
          if (k < hpt) w[k] = *reinterpret_cast<const float4*>(e + (hg + k * hgs) * ts + j);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const float v = staged_one<F16>(slot, j + jj, hd, d);
#pragma unroll
          for (int k = 0; k < G; ++k) {
            if (k < hpt) {
              const float x = jj == 0 ? w[k].x : jj == 1 ? w[k].y : jj == 2 ? w[k].z : w[k].w;
              o[k] = __fmaf_rn(x, v, o[k]);
              if (lsum) l[k] = __fadd_rn(l[k], x);
            }
          }
        }
      }
      for (; j < cn; ++j) {
        const float v = staged_one<F16>(slot, j, hd, d);
#pragma unroll
        for (int k = 0; k < G; ++k) {
          if (k < hpt) {
            const float x = e[(hg + k * hgs) * ts + j];
            o[k] = __fmaf_rn(x, v, o[k]);
            if (lsum) l[k] = __fadd_rn(l[k], x);
          }
        }
      }
    }
    __syncthreads();  // slot c % nslot is refilled by the next iteration
  }
  FOX_ATTN_MARK(6);
  if (vact) {
#pragma unroll
    for (int k = 0; k < G; ++k) {
      if (k < hpt) {
        const int h = hg + k * hgs;
        m.part[h * hd + d] = o[k];
        if (d == 0) s_l[h] = l[k];
      }
    }
  }
}

// The merge of the cluster's tiles: every CTA forms M, the weights and L of
// every head from the tiles' max and sum (read from their CTAs' shared
// memory), then CTA `rank` takes its share [i0, i1) of the G * hd outputs.
template <int G>
FOX_DEV void attn_merge(const TileArgs& a, const TileSmem& m, int g, int nt) {
  __shared__ float s_mt[ATTN_TILE_MAX][ATTN_TILE_GQA], s_lt[ATTN_TILE_MAX][ATTN_TILE_GQA];
  __shared__ float s_w[ATTN_TILE_MAX][ATTN_TILE_GQA], s_M[ATTN_TILE_GQA], s_L[ATTN_TILE_GQA];
  const int tid = threadIdx.x, hd = a.hd;
  const unsigned rank = cluster_ctarank();
  const int th = tid / G, hh = tid - th * G;  // (tile, head) of the first G * nt threads
  if (tid < G * nt) {
    s_mt[th][hh] = cluster_peer(m.ml, th)[hh];
    s_lt[th][hh] = cluster_peer(m.ml + 32, th)[hh];
  }
  __syncthreads();
  if (tid < G) {
    float M = -CUDART_INF_F;
    for (int t = 0; t < nt; ++t) M = fmaxf(M, s_mt[t][tid]);
    s_M[tid] = M;
  }
  __syncthreads();
  if (tid < G * nt) s_w[th][hh] = expf_up(__fsub_rn(s_mt[th][hh], s_M[hh]));
  __syncthreads();
  if (tid < G) {
    float L = 0.0f;
    for (int t = 0; t < nt; ++t) L = __fmaf_rn(s_lt[t][tid], s_w[t][tid], L);
    s_L[tid] = L;
  }
  __syncthreads();
  const int total = G * hd, per = (total + (int)gridDim.x - 1) / (int)gridDim.x;
  const int i0 = (int)rank * per, i1 = min(total, i0 + per);
  for (int i = i0 + tid; i < i1; i += blockDim.x) {
    const int h = i / hd;
    float ov[ATTN_TILE_MAX];
#pragma unroll
    for (int t = 0; t < ATTN_TILE_MAX; ++t) ov[t] = t < nt ? cluster_peer(m.part, t)[i] : 0.0f;
    float O = 0.0f;
#pragma unroll
    for (int t = 0; t < ATTN_TILE_MAX; ++t)
      if (t < nt) O = __fmaf_rn(ov[t], s_w[t][h], O);
    __stcg(a.out + (uint32_t)g * G * hd + i, __fdiv_rn(O, s_L[h]));
  }
}

// Tile attention (AttnParams, ops.cuh): grid (nt, n_kv, n_seq) in clusters
// of nt CTAs (the tiles of one KV head of one sequence). Sequence z reads its
// position at *pos_list[z] (or *pos), its q and output at z * seq_stride,
// and its caches at k_list[z] / v_list[z] + layer_off (or kcache / vcache),
// paged through table_list[z] (or kv_table) when given.
// Under programmatic launch (the decode step, right after the q|k|v kernel
// that writes q and position P - 1) the older rows of the first chunk are
// staged before griddepcontrol.wait; q and the newest row are read after it.
template <int DPL, bool F16, int G>
__global__ void __launch_bounds__(ATTN_THREADS, DPL <= 4 ? 2 : 1) attention_tile_kernel(const AttnParams k) {
  extern __shared__ __align__(16) float tsm[];
  griddep_launch_dependents();  // the o projection may start streaming its weights
  FOX_ATTN_MARK(0);
  const int t = blockIdx.x, g = blockIdx.y, z = blockIdx.z;
  TileArgs a;
  a.q = k.q + (size_t)z * k.seq_stride;
  a.out = k.out + (size_t)z * k.seq_stride;
  a.kc = k.k_list ? (const void*)(reinterpret_cast<const uint8_t*>(k.k_list[z]) + k.layer_off) : k.kcache;
  a.vc = k.v_list ? (const void*)(reinterpret_cast<const uint8_t*>(k.v_list[z]) + k.layer_off) : k.vcache;
  a.table = k.table_list ? k.table_list[z] : k.kv_table;
  a.n_ctx = k.n_ctx; a.n_kv = k.n_kv; a.hd = k.hd; a.nt = k.nt;
  a.P = (k.pos_list ? *k.pos_list[z] : *k.pos) + 1;
  a.scale = k.scale;
  const int T = attn_tile_len(a.P, a.nt), nt = (a.P + T - 1) / T;
  const TileSmem m = tile_smem(tsm, k.n_ctx, k.nt, G, k.hd, F16 ? 1 : 0, k.stage_rows, k.stage_slots);
  const bool live = t < nt;  // CTAs past the last tile only join the cluster's barriers
  if (live) attn_tile_stage0<F16>(a, m, g, t);
  griddep_wait();
  FOX_ATTN_MARK(9);
  if (live) attn_tile<DPL, F16, G>(a, m, g, t);
  cluster_sync();  // every tile's values are in its CTA's shared memory
  FOX_ATTN_MARK(7);
  attn_merge<G>(a, m, g, nt);
  cluster_sync();  // no CTA leaves while another reads its shared memory
  FOX_ATTN_MARK(8);
}

}  // namespace fox
