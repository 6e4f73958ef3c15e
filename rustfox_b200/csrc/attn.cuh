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

constexpr int ATTN_THREADS = 256;    // threads of a tile CTA
constexpr int ATTN_TILE_MAX = 8;     // tile target NT: the tiles of a KV head form one portable cluster
constexpr int ATTN_TILE_GQA = 8;     // query heads per KV head

// Tile length for P positions and tile target nt.
__host__ __device__ inline int attn_tile_len(int P, int nt) { return (P + nt - 1) / nt; }

FOX_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
FOX_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
FOX_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
FOX_DEV void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

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

// K/V rows of one KV head staged in shared memory, ch rows at a time.
struct TileStage {
  uint8_t* k;   // ch rows of K
  uint8_t* v;   // ch rows of V
  int ch;
};

// Where KV head g's positions of one sequence and layer live: the cache
// base, and its block table when paged (common.cuh kv_row).
struct KvHead {
  const uint8_t* base;
  const int* table;
  int n_ctx, n_kv, g, rb;  // rb: row bytes
  FOX_DEV const uint8_t* row(int pos) const { return base + kv_row(table, n_ctx, n_kv, g, pos) * rb; }
};

// Positions [r0, r1) of a head into buf, position r at (r - r0) * rb,
// except position `skip`; asynchronous (cp.async, L2 only), one commit group.
FOX_DEV void stage_rows(uint8_t* buf, const KvHead& kv, int r0, int r1, int skip) {
  const int per_row = kv.rb >> 4, pieces = (r1 - r0) * per_row;
  for (int i = threadIdx.x; i < pieces; i += blockDim.x) {
    const int row = i / per_row;
    if (r0 + row == skip) continue;
    cp_async16(buf + (uint32_t)i * 16, kv.row(r0 + row) + (uint32_t)(i - row * per_row) * 16);
  }
  cp_async_commit();
}

// Row r of a staged chunk as floats (DPL elements from element e0).
template <int DPL, bool F16>
FOX_DEV void staged_row(const uint8_t* buf, int r, int hd, int e0, float* v) {
  if (F16) {
    const __half* p = reinterpret_cast<const __half*>(buf) + (size_t)r * hd + e0;
#pragma unroll
    for (int i = 0; i < DPL; i += 2) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(p + i));
      v[i] = f.x;
      if (i + 1 < DPL) v[i + 1] = f.y;
    }
  } else {
    const float* p = reinterpret_cast<const float*>(buf) + (size_t)r * hd + e0;
#pragma unroll
    for (int i = 0; i < DPL; ++i) v[i] = p[i];
  }
}

// Scores of 16 rows (r0.., at most `valid` of them) of a staged chunk for one
// query head: lane l forms the partial over its hd/32 dimensions for each
// row, then a butterfly reduce-scatter (offsets 16, 8, 4, 2) and a last
// exchange at offset 1 leave row r0 + (lane >> 1)'s dot in lanes 2k, 2k+1.
// Every add pairs the same lane partials as an xor all-reduce (16, 8, 4, 2,
// 1) does, so each dot is the all-reduce's value bit for bit, with 16
// exchanges for 16 rows instead of 80.
template <int DPL, bool F16>
FOX_DEV float dot16(const uint8_t* buf, int r0, int valid, int hd, const float* qh, int lane) {
  float q[DPL];
#pragma unroll
  for (int e = 0; e < DPL; ++e) q[e] = qh[lane * DPL + e];
  float P[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    P[i] = 0.0f;
    if (i < valid) {
      float k[DPL];
      staged_row<DPL, F16>(buf, r0 + i, hd, lane * DPL, k);
      float d = __fmul_rn(q[0], k[0]);
#pragma unroll
      for (int e = 1; e < DPL; ++e) d = __fmaf_rn(q[e], k[e], d);
      P[i] = d;
    }
  }
#pragma unroll
  for (int o = 16, m = 16; o >= 2; o >>= 1, m >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < m / 2; ++i) {
      const float send = up ? P[i] : P[i + m / 2];
      const float keep = up ? P[i + m / 2] : P[i];
      P[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
    }
  }
  return __fadd_rn(P[0], __shfl_xor_sync(0xffffffffu, P[0], 1));
}

// Shared memory of a tile CTA (floats unless noted):
//   sc    G * Tmax   scores, then weights
//   q     G * hd     the group's query heads
//   ml    64         per-head max [0, 32), sum [32, 64); the merge's w [32..)
//   part  G * hd     this tile's unnormalised outputs (read by the cluster)
//   K, V  2 * ch * row bytes  staged rows
struct TileSmem {
  float* sc;
  float* q;
  float* ml;
  float* part;
  TileStage st;
};

inline size_t attn_tile_smem_bytes(int n_ctx, int nt, int gqa, int hd, int kv_f16, int ch) {
  const size_t tmax = (size_t)attn_tile_len(n_ctx, nt);
  const size_t floats = ((size_t)gqa * tmax + 3) / 4 * 4 + (size_t)gqa * hd + 64 + (size_t)gqa * hd;
  return floats * 4 + 2 * (size_t)ch * hd * (kv_f16 ? 2 : 4);
}

FOX_DEV TileSmem tile_smem(float* base, int n_ctx, int nt, int gqa, int hd, int kv_f16, int ch) {
  TileSmem m;
  const int tmax = attn_tile_len(n_ctx, nt);
  m.sc = base;
  m.q = base + (gqa * tmax + 3) / 4 * 4;
  m.ml = m.q + gqa * hd;
  m.part = m.ml + 64;
  m.st.k = reinterpret_cast<uint8_t*>(m.part + gqa * hd);
  m.st.v = m.st.k + (uint32_t)ch * hd * (kv_f16 ? 2 : 4);
  m.st.ch = ch;
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

// The first chunk of tile t of group g, K then V (two commit groups),
// without the newest position P - 1: everything this tile reads that
// earlier steps wrote, so it may be issued before griddepcontrol.wait.
template <bool F16>
FOX_DEV void attn_tile_stage0(const TileArgs& a, const TileStage& st, int g, int t) {
  const int T = attn_tile_len(a.P, a.nt), j0 = t * T, n = min(T, a.P - j0);
  const int rb = a.hd * (F16 ? 2 : 4);
  const int c1 = j0 + min(n, st.ch);
  stage_rows(st.k, a.head(a.kc, g, rb), j0, c1, a.P - 1);
  stage_rows(st.v, a.head(a.vc, g, rb), j0, c1, a.P - 1);
}

// Tile t of KV group g (after attn_tile_stage0): every query head's max,
// sum and unnormalised output into the CTA's shared memory (ml, part).
template <int DPL, bool F16, int G>
FOX_DEV void attn_tile(const TileArgs& a, const TileSmem& m, int g, int t) {
  const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nth >> 5;
  const int T = attn_tile_len(a.P, a.nt);
  const int j0 = t * T, n = min(T, a.P - j0);
  const int hd = a.hd, ch = m.st.ch;
  const int rb = hd * (F16 ? 2 : 4);
  const KvHead kh = a.head(a.kc, g, rb), vh = a.head(a.vc, g, rb);
  const int newest = a.P - 1;
  float* sc = m.sc;
  float* s_m = m.ml;        // [G]
  float* s_l = m.ml + 32;   // [G]
  FOX_ATTN_MARK(1);
  for (int i = tid; i < G * hd; i += nth) m.q[i] = __ldcg(a.q + (uint32_t)g * G * hd + i);
  // the newest row into the first chunk (staging left it out)
  const bool has_newest = newest >= j0 && newest < j0 + min(n, ch);
  auto newest_row = [&](uint8_t* buf, const KvHead& src) {
    if (has_newest)
      for (int i = tid; i < (rb >> 2); i += nth)
        reinterpret_cast<uint32_t*>(buf + (uint32_t)(newest - j0) * rb)[i] =
            __ldcg(reinterpret_cast<const unsigned int*>(src.row(newest)) + i);
  };
  for (int c0 = j0; c0 < j0 + n; c0 += ch) {
    const int c1 = min(j0 + n, c0 + ch), cn = c1 - c0;
    if (c0 == j0) {
      cp_async_wait_one();  // chunk 0's K (its V may still be in flight)
      newest_row(m.st.k, kh);
    } else {
      stage_rows(m.st.k, kh, c0, c1, -1);
      cp_async_wait_all();
    }
    __syncthreads();
    FOX_ATTN_MARK(2);
    // tasks: (group of 16 rows, query head)
    const int groups = (cn + 15) >> 4;
    for (int task = warp; task < groups * G; task += nw) {
      const int r0 = (task / G) * 16, h = task % G;
      const float d = dot16<DPL, F16>(m.st.k, r0, cn - r0, hd, m.q + h * hd, lane);
      const int r = r0 + (lane >> 1);
      if (!(lane & 1) && r < cn) sc[h * T + (c0 - j0) + r] = __fmul_rn(d, a.scale);
    }
    __syncthreads();  // the buffer is refilled by the next chunk
  }
  FOX_ATTN_MARK(3);
  for (int h = warp; h < G; h += nw) {
    float mx = -CUDART_INF_F;
    for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[h * T + j]);
    mx = warp_max(mx);
    if (lane == 0) s_m[h] = mx;
  }
  __syncthreads();
  for (int i = tid; i < G * n; i += nth) {
    const int h = i / n, j = i - h * n;
    sc[h * T + j] = expf_up(__fsub_rn(sc[h * T + j], s_m[h]));
  }
  __syncthreads();
  FOX_ATTN_MARK(4);
  if (tid < G) {
    float l = 0.0f;
    for (int j = 0; j < n; ++j) l = __fadd_rn(l, sc[tid * T + j]);
    s_l[tid] = l;
  }
  // thread (d, hg) holds the sums of heads hg, hg + hgs, ... (hpt of them),
  // each over the positions in order
  const int hgs = max(1, min(G, nth / hd));
  const int hpt = G / hgs;
  const int d = tid % hd, hg = tid / hd;
  const bool sums = hg < hgs;
  float o[G];
#pragma unroll
  for (int k = 0; k < G; ++k) o[k] = 0.0f;
  for (int c0 = j0; c0 < j0 + n; c0 += ch) {
    const int c1 = min(j0 + n, c0 + ch), cn = c1 - c0;
    if (c0 == j0) {
      cp_async_wait_all();
      newest_row(m.st.v, vh);
    } else {
      __syncthreads();
      stage_rows(m.st.v, vh, c0, c1, -1);
      cp_async_wait_all();
    }
    __syncthreads();
    FOX_ATTN_MARK(5);
    if (sums) {
      const float* e = sc + (c0 - j0) + hg * T;
      const int estep = hgs * T;
#pragma unroll 4
      for (int j = 0; j < cn; ++j) {
        const float v = F16 ? __half2float(reinterpret_cast<const __half*>(m.st.v)[j * hd + d])
                            : reinterpret_cast<const float*>(m.st.v)[j * hd + d];
#pragma unroll
        for (int k = 0; k < G; ++k)
          if (k < hpt) o[k] = __fmaf_rn(e[k * estep + j], v, o[k]);
      }
    }
  }
  FOX_ATTN_MARK(6);
  if (sums) {
#pragma unroll
    for (int k = 0; k < G; ++k)
      if (k < hpt) m.part[(hg + k * hgs) * hd + d] = o[k];
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
__global__ void __launch_bounds__(ATTN_THREADS, 1) attention_tile_kernel(const AttnParams k) {
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
  const TileSmem m = tile_smem(tsm, k.n_ctx, k.nt, G, k.hd, F16 ? 1 : 0, k.stage_rows);
  const bool live = t < nt;  // CTAs past the last tile only join the cluster's barriers
  if (live) attn_tile_stage0<F16>(a, m.st, g, t);
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
