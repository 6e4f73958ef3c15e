// The decode step of a single-GPU ternary model as ONE persistent kernel
// (sm_100a): embedding, then per layer q|k|v (+RMSNorm, RoPE, K/V write),
// attention, o (+residual), gate|up (+RMSNorm, SwiGLU) and down (+residual),
// upstream src/forward.c:295-399 for one token.
//
// One CTA per SM, launched cooperatively so that every CTA is resident. The
// phases are separated by grid barriers (a counter in global memory, waits
// bounded by %globaltimer). Everything a phase can do before its inputs exist
// happens before the barrier it waits at.
//
// Weights. Each CTA owns the same run of whole units of every layer matrix
// as the resident-slice kernel (slice.cuh, units of U rows, CTA c owns units
// [c * per, (c + 1) * per)). The runs of all phases of all layers form one
// sequence of pieces (a piece is a run of whole units that fits one slot).
// Thread 0 keeps n_slots pieces in flight as bulk asynchronous copies
// (cp.async.bulk into shared-memory slots, counted on one mbarrier per slot)
// and issues the next piece into a slot as soon as its piece is consumed.
// The weight stream therefore runs ahead across phases and barriers, and is
// never tied to a kernel boundary.
//
// The GEMV arithmetic is the resident-slice kernel's: lanes l and l+16 split a
// 256 block, the int32 halves meet through a shuffle, and one thread per row
// folds the row's block terms in upstream's order (src/gemv.c:54-97,
// src/ternary.c:177-188,226-246), so every row is bit-identical to it.
//
// Quantiser inputs. The q|k|v and gate|up prologues norm the residual and
// take its absmax inside the CTA (upstream src/ops.c:7-22, src/gemv.c:11-42).
// The o and down inputs are produced by this kernel: every producing CTA
// publishes the absmax of what it wrote, and a consumer takes the largest of
// those slots (max is exact in any order), so it quantises in one pass.
//
// Attention (upstream src/forward.c:222-257) has two forms.
//   exact   one CTA per query head in upstream's serial order (the parity
//           mode; also attention_exact_kernel in ops.cuh);
//   tiles   the positions 0..P-1 are cut into tiles of T positions,
//           T = 32 * ceil(P / (32 * NT)) for the model's tile target NT, so
//           there are at most NT tiles. Per KV head g and tile t, a CTA forms
//           for each query head of the group:
//             s_j = dot(q, k_j) * scale, the dot as 32 lane partials over
//                   hd/32 dims each (q0*k0, then fmaf in dimension order)
//                   summed by an xor butterfly (16, 8, 4, 2, 1);
//             m_t = max_j s_j;  e_j = expf(s_j - m_t);
//             l_t = sum_j e_j (ascending j);
//             o_t = sum_j fmaf(e_j, v_j, .) (ascending j, from 0).
//           The last CTA of head g merges the tiles:
//             M = max_t m_t;  w_t = expf(m_t - M);
//             L = sum_t fmaf(l_t, w_t, .);  O = sum_t fmaf(o_t, w_t, .)
//             (ascending t, from 0);  out = O / L.
//           attention_tile_kernel below computes the same values one launch
//           per attention (prompt chunks, batches, tensor-parallel shards).
//           The oracle restates this order (or_ctx with a tile target).
#pragma once

#include <math_constants.h>

#include "ops.cuh"
#include "slice.cuh"

namespace fox {

constexpr int LOOP_THREADS = 512;
constexpr int LOOP_PAIRS = LOOP_THREADS / 2;
constexpr int LOOP_MAX_KR = 4;       // float4 rounds per thread of the residual: n_embd <= 8192
constexpr int LOOP_MAX_GQA = 8;
constexpr int ATTN_TILE_MAX = 64;    // tile target NT is at most this
constexpr unsigned LOOP_COPY_CHUNK = 32768;

// One layer matrix as the loop kernel walks it.
struct LoopMat {
  const uint8_t* w;    // packed slice layout (pack.cuh, units of U rows)
  int n_rows, nb, U, ushift;
  int units, per;      // CTA c owns units [c * per, min(units, (c + 1) * per))
  int unit_bytes;
  int piece_units;     // units per piece (piece_units * unit_bytes <= slot bytes)
};

enum { LM_QKV = 0, LM_O = 1, LM_GU = 2, LM_DOWN = 3 };

struct LoopLayer {
  LoopMat m[4];
  const float* attn_norm;
  const float* ffn_norm;
  void* kc;  // this layer's caches [n_kv][n_ctx][hd]
  void* vc;
};

struct LoopParams {
  const LoopLayer* layers;
  int n_layer, n_embd, n_ff, hd, n_head, n_kv, nq, nkv, n_ctx, kv_f16;
  float eps, attn_scale;
  int attn_exact, attn_nt;
  const float* rope_cos;
  const float* rope_sin;
  const int* pos;
  const uint32_t* token;
  const uint8_t* embd;
  int embd_type;
  long embd_rb;
  float* x;        // residual [n_embd]
  float* q;        // roped q [nq]
  float* att;      // attention output [nq]
  float* h;        // SwiGLU output [n_ff]
  float* part;     // tile partials [n_kv][NT][gqa][hd + 2]
  unsigned* cnt;   // [n_kv] tiles done (0 between launches)
  float* amax_att; // [max(n_head, n_kv)] absmax of what each attention producer wrote
  float* amax_h;   // [grid] absmax of each CTA's SwiGLU outputs
  unsigned* bar;   // [0] arrivals, [1] arrivals before this launch
  int* err;        // 3: a grid barrier gave up; 1: a weight copy gave up
  float* trace;    // optional [(n_layer + 1) * n_embd]: x after the embedding and each layer
  int n_slots, slot_bytes;
  int attn_ch;     // K/V rows per staged chunk of the attention
  int ring_off, xq_off, part_off, vals_off, scr_off, scr_bytes, bar_off, red_off;
};

// ---- grid barrier ----------------------------------------------------------

FOX_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
FOX_DEV unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
FOX_DEV void red_release_gpu_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Every CTA arrives once; returns once the counter reaches target, or false
// after about a second (then the error word is set). The CTA's writes are
// ordered before thread 0's release by the block barrier (a release is
// cumulative), and the acquire that sees the count orders the reads after
// it; the readers of another CTA's data use L2 loads (ld.cg).
FOX_DEV bool grid_barrier(unsigned* bar, unsigned target, int* err, int* ok_sh) {
  __syncthreads();
  if (threadIdx.x == 0) {
    red_release_gpu_add(bar, 1u);
    int ok = 0;
    const uint64_t t0 = globaltimer_ns();
    for (int i = 0;; ++i) {
      if ((int)(ld_acquire_gpu(bar) - target) >= 0) { ok = 1; break; }
      if ((i & 63) == 63 && globaltimer_ns() - t0 > 1000000000ull) break;
      if (i > 64) __nanosleep(32);
    }
    if (!ok && err) atomicExch(err, 3);
    *ok_sh = ok;
  }
  __syncthreads();
  return *ok_sh != 0;
}

// ---- tile attention --------------------------------------------------------

// Tile length for P positions and tile target nt.
__host__ __device__ inline int attn_tile_len(int P, int nt) {
  const int per = (P + nt - 1) / nt;
  return ((per + 31) / 32) * 32;
}

template <int DPL>
FOX_DEV void load_row(const void* cache, bool f16, size_t off, float* v) {
  if (f16) {
    const __half* p = reinterpret_cast<const __half*>(cache) + off;
    if (DPL == 4) {
      uint2 r;
      asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else if (DPL == 2) {
      unsigned r;
      asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(r) : "l"(p));
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r));
      v[0] = a.x; v[1] = a.y;
    } else {
#pragma unroll
      for (int i = 0; i < DPL; ++i) v[i] = __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short*>(p) + i)));
    }
  } else {
    const float* p = reinterpret_cast<const float*>(cache) + off;
#pragma unroll
    for (int i = 0; i < DPL; ++i) v[i] = __ldcg(p + i);
  }
}

FOX_DEV float load_elem(const void* cache, bool f16, size_t off) {
  if (f16) return __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short*>(cache) + off)));
  return __ldcg(reinterpret_cast<const float*>(cache) + off);
}

struct TileArgs {
  const float* q;     // the group's query heads start at q + g * gqa * hd
  const void* kc;     // [n_kv][n_ctx][hd] of this layer (and sequence)
  const void* vc;
  float* out;         // [n_head * hd]
  float* part;        // [n_kv][NT][gqa][hd + 2]
  unsigned* cnt;      // [n_kv]
  float* amax;        // [n_kv] absmax of each group's outputs, or null
  int f16, n_ctx, hd, gqa, nt, P;
  float scale;
};

// Floats of the tile attention's small scratch (per-head max and sum, then
// the merge's per-tile values), a multiple of 4 so what follows stays
// 16-byte aligned.
__host__ __device__ inline int attn_sm_floats(int nt, int gqa) {
  const int n = 3 * nt * gqa + 2 * gqa;
  return ((n < 64 ? 64 : n) + 3) / 4 * 4;
}

FOX_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
FOX_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
FOX_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
FOX_DEV void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// K/V rows of one KV head staged in shared memory, ch rows at a time.
struct TileStage {
  uint8_t* k;   // ch rows of K
  uint8_t* v;   // ch rows of V
  int ch;
};

// Rows [r0, r1) of a head's cache (row bytes rb) into buf, row r at
// (r - r0) * rb, except row `skip`; asynchronous (cp.async, L2 only), one
// commit group.
FOX_DEV void stage_rows(uint8_t* buf, const uint8_t* head, int rb, int r0, int r1, int skip) {
  const int per_row = rb >> 4, pieces = (r1 - r0) * per_row;
  for (int i = threadIdx.x; i < pieces; i += blockDim.x) {
    const int row = i / per_row;
    if (r0 + row == skip) continue;
    cp_async16(buf + (size_t)i * 16, head + (size_t)r0 * rb + (size_t)i * 16);
  }
  cp_async_commit();
}

// The first chunk of tile t of group g, K then V (two commit groups),
// without the newest position P - 1: everything this tile reads that
// earlier steps wrote. It may be issued before the step's q and newest K/V
// row exist (before a grid barrier, or before griddepcontrol.wait).
FOX_DEV void attn_tile_stage0(const TileArgs& a, const TileStage& st, int g, int t) {
  const int T = attn_tile_len(a.P, a.nt), j0 = t * T, n = min(T, a.P - j0);
  const int rb = a.hd * (a.f16 ? 2 : 4);
  const size_t head = (size_t)g * a.n_ctx * rb;
  const int c1 = j0 + min(n, st.ch);
  stage_rows(st.k, reinterpret_cast<const uint8_t*>(a.kc) + head, rb, j0, c1, a.P - 1);
  stage_rows(st.v, reinterpret_cast<const uint8_t*>(a.vc) + head, rb, j0, c1, a.P - 1);
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
  float P[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    P[i] = 0.0f;
    if (i < valid) {
      float k[DPL];
      staged_row<DPL, F16>(buf, r0 + i, hd, lane * DPL, k);
      float d = __fmul_rn(qh[0], k[0]);
#pragma unroll
      for (int e = 1; e < DPL; ++e) d = __fmaf_rn(qh[e], k[e], d);
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

// Tile t of KV group g, after attn_tile_stage0 for it: the partials of every
// query head of the group. The shared scratch holds gqa * T floats (scores,
// then weights) and attn_sm_floats more; K and V pass through st in chunks
// of st.ch rows. q and the newest row are read here (they may come from the
// work just before).
template <int DPL, bool F16>
FOX_DEV void attn_tile_t(const TileArgs& a, const TileStage& st, int g, int t, float* sc, float* sm) {
  const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nth >> 5;
  const int T = attn_tile_len(a.P, a.nt);
  const int j0 = t * T, n = min(T, a.P - j0);
  const int hd = a.hd, gqa = a.gqa;
  const int rb = hd * (F16 ? 2 : 4);
  const uint8_t* kh = reinterpret_cast<const uint8_t*>(a.kc) + (size_t)g * a.n_ctx * rb;
  const uint8_t* vh = reinterpret_cast<const uint8_t*>(a.vc) + (size_t)g * a.n_ctx * rb;
  const int newest = a.P - 1;
  float qv[LOOP_MAX_GQA][DPL];
#pragma unroll
  for (int h = 0; h < LOOP_MAX_GQA; ++h)
#pragma unroll
    for (int i = 0; i < DPL; ++i)
      qv[h][i] = h < gqa ? __ldcg(a.q + ((size_t)g * gqa + h) * hd + lane * DPL + i) : 0.0f;
  // the newest row into the first chunk (staging left it out)
  auto newest_row = [&](uint8_t* buf, const uint8_t* src) {
    if (newest >= j0 && newest < j0 + min(n, st.ch))
      for (int i = tid; i < (rb >> 2); i += nth)
        reinterpret_cast<uint32_t*>(buf + (size_t)(newest - j0) * rb)[i] =
            __ldcg(reinterpret_cast<const unsigned int*>(src + (size_t)newest * rb) + i);
  };
  for (int c0 = j0; c0 < j0 + n; c0 += st.ch) {
    const int c1 = min(j0 + n, c0 + st.ch), cn = c1 - c0;
    if (c0 == j0) {
      cp_async_wait_one();  // chunk 0's K (its V may still be in flight)
      newest_row(st.k, kh);
    } else {
      stage_rows(st.k, kh, rb, c0, c1, -1);
      cp_async_wait_all();
    }
    __syncthreads();
    // tasks: (group of 16 rows, query head)
    const int groups = (cn + 15) >> 4;
    for (int task = warp; task < groups * gqa; task += nw) {
      const int r0 = (task / gqa) * 16, h = task - (task / gqa) * gqa;
      float qh[DPL];
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        qh[i] = qv[0][i];
#pragma unroll
        for (int hh = 1; hh < LOOP_MAX_GQA; ++hh)
          if (hh == h) qh[i] = qv[hh][i];
      }
      const float d = dot16<DPL, F16>(st.k, r0, cn - r0, hd, qh, lane);
      const int r = r0 + (lane >> 1);
      if (!(lane & 1) && r < cn) sc[h * T + (c0 - j0) + r] = __fmul_rn(d, a.scale);
    }
    __syncthreads();  // the buffer is refilled by the next chunk
  }
  float* s_m = sm;          // [gqa]
  float* s_l = sm + 32;     // [gqa]
  for (int h = warp; h < gqa; h += nw) {
    float mx = -CUDART_INF_F;
    for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[h * T + j]);
    mx = warp_max(mx);
    if (lane == 0) s_m[h] = mx;
  }
  __syncthreads();
  for (int i = tid; i < gqa * n; i += nth) {
    const int h = i / n, j = i - h * n;
    sc[h * T + j] = expf_cr(__fsub_rn(sc[h * T + j], s_m[h]));
  }
  __syncthreads();
  if (tid < gqa) {
    float l = 0.0f;
    for (int j = 0; j < n; ++j) l = __fadd_rn(l, sc[tid * T + j]);
    s_l[tid] = l;
  }
  // thread (d, hg) holds the sums of heads hg, hg + hgs, ...: each in order
  const int hgs = max(1, min(gqa, nth / hd));
  const int d = tid % hd, hg = tid / hd;
  const bool sums = hg < hgs;
  float o[LOOP_MAX_GQA];
#pragma unroll
  for (int h = 0; h < LOOP_MAX_GQA; ++h) o[h] = 0.0f;
  for (int c0 = j0; c0 < j0 + n; c0 += st.ch) {
    const int c1 = min(j0 + n, c0 + st.ch), cn = c1 - c0;
    if (c0 == j0) {
      cp_async_wait_all();
      newest_row(st.v, vh);
    } else {
      __syncthreads();
      stage_rows(st.v, vh, rb, c0, c1, -1);
      cp_async_wait_all();
    }
    __syncthreads();
    if (sums) {
      const float* e = sc + (c0 - j0);
#pragma unroll 4
      for (int j = 0; j < cn; ++j) {
        const float v = F16 ? __half2float(reinterpret_cast<const __half*>(st.v)[(size_t)j * hd + d])
                            : reinterpret_cast<const float*>(st.v)[(size_t)j * hd + d];
#pragma unroll
        for (int h = 0; h < LOOP_MAX_GQA; ++h)
          if (h < gqa && h % hgs == hg) o[h] = __fmaf_rn(e[h * T + j], v, o[h]);
      }
    }
  }
  float* part = a.part + ((size_t)g * a.nt + t) * gqa * (hd + 2);
  if (sums) {
#pragma unroll
    for (int h = 0; h < LOOP_MAX_GQA; ++h)
      if (h < gqa && h % hgs == hg) __stcg(part + (size_t)h * (hd + 2) + d, o[h]);
  }
  __syncthreads();
  if (tid < gqa) {
    __stcg(part + (size_t)tid * (hd + 2) + hd, s_m[tid]);
    __stcg(part + (size_t)tid * (hd + 2) + hd + 1, s_l[tid]);
  }
}

template <int DPL>
FOX_DEV void attn_tile(const TileArgs& a, const TileStage& st, int g, int t, float* sc, float* sm) {
  if (a.f16) attn_tile_t<DPL, true>(a, st, g, t, sc, sm);
  else attn_tile_t<DPL, false>(a, st, g, t, sc, sm);
}

constexpr int MERGE_BATCH = 32;  // tile partials a merging thread requests at once

// After attn_tile: the CTA that completes KV group g's last tile merges all
// its tiles into the output (and publishes the absmax of what it wrote).
// The scratch holds attn_sm_floats(nt, gqa) floats.
FOX_DEV void attn_merge_tiles(const TileArgs& a, int g, float* sm, float* red) {
  __shared__ int last_sh;
  const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nth >> 5;
  const int hd = a.hd, gqa = a.gqa;
  const int T = attn_tile_len(a.P, a.nt), nt = (a.P + T - 1) / T;
  __threadfence();
  __syncthreads();
  if (tid == 0) last_sh = atomicAdd(a.cnt + g, 1u) == (unsigned)(nt - 1);
  __syncthreads();
  if (!last_sh) return;
  __threadfence();
  const float* base = a.part + (size_t)g * a.nt * gqa * (hd + 2);
  float* s_m = sm;                      // [nt][gqa]
  float* s_l = sm + a.nt * gqa;         // [nt][gqa]
  float* s_w = sm + 2 * a.nt * gqa;     // [nt][gqa]
  float* s_M = sm + 3 * a.nt * gqa;     // [gqa]
  float* s_L = s_M + gqa;               // [gqa]
  // the first batch of this thread's first (head, dimension) partials is
  // requested with the small values
  const int h0 = tid / hd, d0 = tid - h0 * hd;
  const bool first = tid < gqa * hd;
  float ov[MERGE_BATCH];
#pragma unroll
  for (int t = 0; t < MERGE_BATCH; ++t)
    ov[t] = (first && t < nt) ? __ldcg(base + ((size_t)t * gqa + h0) * (hd + 2) + d0) : 0.0f;
  for (int i = tid; i < nt * gqa; i += nth) {
    const float* pt = base + (size_t)i * (hd + 2);
    s_m[i] = __ldcg(pt + hd);
    s_l[i] = __ldcg(pt + hd + 1);
  }
  __syncthreads();
  for (int h = warp; h < gqa; h += nw) {
    float M = -CUDART_INF_F;
    for (int t = lane; t < nt; t += 32) M = fmaxf(M, s_m[t * gqa + h]);
    M = warp_max(M);
    if (lane == 0) s_M[h] = M;
  }
  __syncthreads();
  for (int i = tid; i < nt * gqa; i += nth) s_w[i] = expf_cr(__fsub_rn(s_m[i], s_M[i % gqa]));
  __syncthreads();
  if (tid < gqa) {
    float L = 0.0f;
    for (int t = 0; t < nt; ++t) L = __fmaf_rn(s_l[t * gqa + tid], s_w[t * gqa + tid], L);
    s_L[tid] = L;
  }
  __syncthreads();
  float am = 0.0f;
  for (int i = tid; i < gqa * hd; i += nth) {
    const int h = i / hd, d = i - h * hd;
    float O = 0.0f;
    for (int t0 = 0; t0 < nt; t0 += MERGE_BATCH) {
      if (i != tid || t0 > 0) {
#pragma unroll
        for (int t = 0; t < MERGE_BATCH; ++t)
          ov[t] = t0 + t < nt ? __ldcg(base + ((size_t)(t0 + t) * gqa + h) * (hd + 2) + d) : 0.0f;
      }
#pragma unroll
      for (int t = 0; t < MERGE_BATCH; ++t)
        if (t0 + t < nt) O = __fmaf_rn(ov[t], s_w[(t0 + t) * gqa + h], O);
    }
    const float v = __fdiv_rn(O, s_L[h]);
    __stcg(a.out + ((size_t)g * gqa + h) * hd + d, v);
    am = absmax_acc(am, v);
  }
  if (a.amax) {
    am = block_reduce<float>(am, red, OpMax(), 0.0f);
    if (tid == 0) __stcg(a.amax + g, am);
  }
  if (tid == 0) a.cnt[g] = 0u;
}

// Upstream's serial attention for query head h (src/forward.c:222-257), as
// attention_exact_kernel: the scratch holds P floats. Publishes the head's
// absmax into amax[h] when given.
FOX_DEV void attn_exact_head(const TileArgs& a, int h, float* att, float* red, float* bcast) {
  const int tid = threadIdx.x, nth = blockDim.x, hd = a.hd;
  const int kvh = h / a.gqa, P = a.P;
  const bool f16 = a.f16 != 0;
  const float* qh = a.q + (size_t)h * hd;
  const size_t base = (size_t)kvh * a.n_ctx * hd;
  for (int j = tid; j < P; j += nth) {
    float s = 0.0f;
    for (int d = 0; d < hd; ++d)
      s = __fadd_rn(s, __fmul_rn(__ldcg(qh + d), load_elem(a.kc, f16, base + (size_t)j * hd + d)));
    att[j] = __fmul_rn(s, a.scale);
  }
  __syncthreads();
  float mx = -CUDART_INF_F;
  for (int j = tid; j < P; j += nth) mx = fmaxf(mx, att[j]);
  mx = block_reduce<float>(mx, red, OpMax(), -CUDART_INF_F);
  for (int j = tid; j < P; j += nth) att[j] = expf_cr(__fsub_rn(att[j], mx));
  __syncthreads();
  if (tid == 0) {
    float sum = 0.0f;
    for (int j = 0; j < P; ++j) sum = __fadd_rn(sum, att[j]);
    bcast[0] = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 0.0f;
    bcast[1] = sum > 0.0f ? 1.0f : 0.0f;
  }
  __syncthreads();
  if (bcast[1] != 0.0f)
    for (int j = tid; j < P; j += nth) att[j] = __fmul_rn(att[j], bcast[0]);
  __syncthreads();
  float am = 0.0f;
  for (int d = tid; d < hd; d += nth) {
    float acc = 0.0f;
    for (int j = 0; j < P; ++j)
      acc = __fadd_rn(acc, __fmul_rn(att[j], load_elem(a.vc, f16, base + (size_t)j * hd + d)));
    __stcg(a.out + (size_t)h * hd + d, acc);
    am = absmax_acc(am, acc);
  }
  if (a.amax) {
    am = block_reduce<float>(am, red, OpMax(), 0.0f);
    if (tid == 0) __stcg(a.amax + h, am);
  }
}

// Standalone tile attention (AttnParams, ops.cuh): grid (nt, n_kv, n_seq).
// Sequence z reads its position at *pos_list[z] (or *pos), its q and output
// at z * seq_stride, its caches at k_list[z] / v_list[z] + layer_off (or
// kcache / vcache), and uses the partials and counters of slot z. Under
// programmatic launch (the decode step, right after the q|k|v kernel that
// writes q and position P - 1) the older rows of the first chunk are staged
// before griddepcontrol.wait; q and the newest row are read after it.
constexpr int ATTN_STAGE_ROWS = 64;  // K/V rows per staged chunk of the standalone kernel

template <int DPL>
__global__ void __launch_bounds__(256, 1) attention_tile_kernel(const AttnParams k) {
  extern __shared__ __align__(16) float tsm[];
  __shared__ float red[32];
  griddep_launch_dependents();  // the o projection may start streaming its weights
  const int t = blockIdx.x, g = blockIdx.y, z = blockIdx.z;
  const int gqa = k.n_head / k.n_kv;
  TileArgs a;
  a.q = k.q + (size_t)z * k.seq_stride;
  a.out = k.out + (size_t)z * k.seq_stride;
  a.kc = k.k_list ? (const void*)(reinterpret_cast<const uint8_t*>(k.k_list[z]) + k.layer_off) : k.kcache;
  a.vc = k.v_list ? (const void*)(reinterpret_cast<const uint8_t*>(k.v_list[z]) + k.layer_off) : k.vcache;
  a.part = k.part + (size_t)z * k.n_kv * k.nt * gqa * (k.hd + 2);
  a.cnt = k.counters + (size_t)z * k.n_kv;
  a.amax = nullptr;
  a.f16 = k.kv_f16; a.n_ctx = k.n_ctx; a.hd = k.hd; a.gqa = gqa; a.nt = k.nt;
  a.P = (k.pos_list ? *k.pos_list[z] : *k.pos) + 1;
  a.scale = k.scale;
  const int T = attn_tile_len(a.P, a.nt);
  if (t * T >= a.P) return;
  const int Tmax = attn_tile_len(k.n_ctx, k.nt);
  float* sc = tsm;                                   // gqa * Tmax
  float* sm = tsm + (size_t)gqa * Tmax;              // attn_sm_floats
  TileStage st;
  st.ch = ATTN_STAGE_ROWS;
  st.k = reinterpret_cast<uint8_t*>(sm + attn_sm_floats(k.nt, gqa));
  st.v = st.k + (size_t)st.ch * k.hd * (k.kv_f16 ? 2 : 4);
  attn_tile_stage0(a, st, g, t);
  griddep_wait();
  attn_tile<DPL>(a, st, g, t, sc, sm);
  __syncthreads();
  attn_merge_tiles(a, g, sm, red);
}

// Shared memory of attention_tile_kernel for contexts of n_ctx positions.
inline size_t attn_tile_smem_bytes(int n_ctx, int nt, int gqa, int hd, int kv_f16) {
  const int T = attn_tile_len(n_ctx, nt);
  return ((size_t)gqa * T + (size_t)attn_sm_floats(nt, gqa)) * 4 +
         2 * (size_t)ATTN_STAGE_ROWS * hd * (kv_f16 ? 2 : 4);
}

// ---- the persistent decode step --------------------------------------------

struct PieceCursor { int l, m, k; };

// The next piece of this CTA's weight sequence (layer-major, then phase, then
// piece), or false at the end.
FOX_DEV bool next_piece(const LoopParams& p, int cta, PieceCursor& c, const uint8_t** src, unsigned* bytes) {
  while (c.l < p.n_layer) {
    const LoopMat& M = p.layers[c.l].m[c.m];
    const int u0 = cta * M.per;
    const int nu = max(0, min(M.per, M.units - u0));
    const int np = (nu + M.piece_units - 1) / M.piece_units;
    if (c.k < np) {
      const int pu0 = u0 + c.k * M.piece_units;
      const int pn = min(M.piece_units, u0 + nu - pu0);
      *src = M.w + (size_t)pu0 * M.unit_bytes;
      *bytes = (unsigned)pn * (unsigned)M.unit_bytes;
      ++c.k;
      return true;
    }
    c.k = 0;
    if (++c.m == 4) { c.m = 0; ++c.l; }
  }
  return false;
}

FOX_DEV void issue_piece(uint8_t* dst, const uint8_t* src, unsigned bytes, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, bytes);
  for (unsigned o = 0; o < bytes; o += LOOP_COPY_CHUNK)
    bulk_g2s(dst + o, src + o, min(LOOP_COPY_CHUNK, bytes - o), bar);
}

// Per-CTA state of the loop kernel.
struct LoopState {
  uint8_t* ring;
  uint64_t* full;
  int8_t* xq;
  float* part;
  float* vals;
  float* scr;
  float* red;
  int* flag;          // shared: barrier / wait results
  int consumed;       // pieces consumed (uniform across the CTA)
  int issued;         // thread 0: pieces issued
  PieceCursor cur;    // thread 0: next piece
  unsigned base;      // barrier counter at launch
  int nbar;           // barriers passed
};

// Wait (bounded) for every copy still in flight, so the kernel can exit.
FOX_DEV void drain_copies(const LoopParams& p, LoopState& s) {
  if (threadIdx.x == 0)
    for (int k = s.consumed; k < s.issued; ++k) mbar_wait(s.full + (k % p.n_slots), (k / p.n_slots) & 1);
  __syncthreads();
}

FOX_DEV bool loop_barrier(const LoopParams& p, LoopState& s) {
  ++s.nbar;
  return grid_barrier(p.bar, s.base + (unsigned)(s.nbar * gridDim.x), p.err, s.flag);
}

// x -> RMSNorm (double sum of squares) -> upstream's quantiser, into xq.
// v holds this thread's float4s of x; w this thread's float4s of the norm
// weights. Returns the activation scale.
FOX_DEV float pro_norm(const LoopParams& p, LoopState& s, float4 (&v)[LOOP_MAX_KR],
                       const float4 (&w)[LOOP_MAX_KR], int K) {
  const int tid = threadIdx.x, nth = blockDim.x, K4 = K >> 2;
  double ss = 0.0;
#pragma unroll
  for (int k = 0; k < LOOP_MAX_KR; ++k) {
    if (tid + k * nth < K4)
      ss = ss + (double)v[k].x * (double)v[k].x + (double)v[k].y * (double)v[k].y +
           (double)v[k].z * (double)v[k].z + (double)v[k].w * (double)v[k].w;
  }
  const double sum = block_reduce<double>(ss, reinterpret_cast<double*>(s.red), OpAddD(), 0.0);
  const float scale = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)K), (double)p.eps)));
  float am = 0.0f;
#pragma unroll
  for (int k = 0; k < LOOP_MAX_KR; ++k) {
    if (tid + k * nth < K4) {
      v[k].x = __fmul_rn(__fmul_rn(v[k].x, scale), w[k].x);
      v[k].y = __fmul_rn(__fmul_rn(v[k].y, scale), w[k].y);
      v[k].z = __fmul_rn(__fmul_rn(v[k].z, scale), w[k].z);
      v[k].w = __fmul_rn(__fmul_rn(v[k].w, scale), w[k].w);
      am = absmax_acc(absmax_acc(absmax_acc(absmax_acc(am, v[k].x), v[k].y), v[k].z), v[k].w);
    }
  }
  const float amax = block_reduce<float>(am, s.red + 64, OpMax(), 0.0f);
  const bool nz = amax > 0.0f;
  const float inv = nz ? __fdiv_rn(127.0f, amax) : 0.0f;
#pragma unroll
  for (int k = 0; k < LOOP_MAX_KR; ++k) {
    const int i = (tid + k * nth) * 4;
    if (i < K)
      *reinterpret_cast<uint32_t*>(s.xq + (i >> 8) * XQ_STRIDE + (i & 255)) =
          pack4(quant1(v[k].x, inv), quant1(v[k].y, inv), quant1(v[k].z, inv), quant1(v[k].w, inv));
  }
  __syncthreads();
  return nz ? __fdiv_rn(amax, 127.0f) : 0.0f;
}

// A vector this kernel produced (att or h) -> upstream's quantiser, with the
// absmax taken from its producers' slots. Every warp reduces the slots itself.
FOX_DEV float pro_vec(LoopState& s, const float* src, int K, const float* slots, int n_slots) {
  const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31;
  float am = 0.0f;
  for (int i = lane; i < n_slots; i += 32) am = fmaxf(am, __ldcg(slots + i));
  const float amax = warp_max(am);
  const bool nz = amax > 0.0f;
  const float inv = nz ? __fdiv_rn(127.0f, amax) : 0.0f;
  for (int i4 = tid; i4 < (K >> 2); i4 += nth) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(src) + i4);
    const int i = i4 * 4;
    *reinterpret_cast<uint32_t*>(s.xq + (i >> 8) * XQ_STRIDE + (i & 255)) =
        pack4(quant1(v.x, inv), quant1(v.y, inv), quant1(v.z, inv), quant1(v.w, inv));
  }
  __syncthreads();
  return nz ? __fdiv_rn(amax, 127.0f) : 0.0f;
}

enum { LE_QKV = 0, LE_ADD = 1, LE_SWIGLU = 2 };

// One layer matrix against the quantised input in xq: decode this CTA's run
// piece by piece from the ring, fold each row in upstream's order, apply the
// epilogue. LE_ADD also writes the new residual rows to trace (when given);
// LE_SWIGLU leaves the absmax of its outputs in *am_out (thread 0). Returns
// false if a weight copy gave up.
template <int EPI>
FOX_DEV bool loop_gemv(const LoopParams& p, LoopState& s, const LoopMat& M, float act_scale, int layer,
                       float* trace, float* am_out) {
  using H = HalfW<T_TQ2_0>;
  const int tid = threadIdx.x, nth = blockDim.x, cta = blockIdx.x;
  const int nb = M.nb, U = M.U;
  const int u0 = cta * M.per;
  const int nu = max(0, min(M.per, M.units - u0));
  if (nu == 0) {
    if (EPI == LE_SWIGLU && tid == 0) *am_out = 0.0f;
    return true;
  }
  const int lane = tid & 31, h = lane >> 4;
  const int pair = (tid >> 5) * 16 + (lane & 15);
  const int S = LOOP_PAIRS / nb;
  const bool active = pair < S * nb;
  const int col = active ? pair % nb : 0, slot_r = active ? pair / nb : 0;
  uint32_t xa[H::NX];
  int sx;
  {
    const uint4* x4 = reinterpret_cast<const uint4*>(s.xq + col * XQ_STRIDE) + 8 * h;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 v = x4[i];
      xa[4 * i] = v.x; xa[4 * i + 1] = v.y; xa[4 * i + 2] = v.z; xa[4 * i + 3] = v.w;
    }
    int s4[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < H::NX; ++i) s4[i & 3] = dp4a(0x01010101u, xa[i], s4[i & 3]);
    sx = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  }
  const long cnt = (long)U * nb;
  const int rstride = nb + 1;
  const int np = (nu + M.piece_units - 1) / M.piece_units;
  float am = 0.0f;
  for (int k = 0; k < np; ++k) {
    const int pu0 = u0 + k * M.piece_units;
    const int pn = min(M.piece_units, u0 + nu - pu0);
    const int rows = pn * U;
    const int slot = s.consumed % p.n_slots;
    const bool got = mbar_wait(s.full + slot, (s.consumed / p.n_slots) & 1);
    if (!__syncthreads_and(got)) {
      if (tid == 0 && p.err) atomicExch(p.err, 1);
      return false;
    }
    const uint8_t* sw = s.ring + (size_t)slot * p.slot_bytes;
    const int passes = (rows + S - 1) / S;
    for (int ps = 0; ps < passes; ++ps) {
      const int r = slot_r + ps * S;
      const bool on = active && r < rows;
      int v = 0;
      const int ul = on ? r >> M.ushift : 0, t = on ? (r - ul * U) * nb + col : 0;
      const uint8_t* base = sw + (size_t)ul * M.unit_bytes;
      if (on) v = H::isum(base, cnt, t, h, xa) - sx;
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      if (on && h == 0) s.part[r * rstride + col] = __fmul_rn(H::scale(base, cnt, t), __int2float_rn(v));
    }
    __syncthreads();
    // the slot is free again: the next piece of the sequence goes into it
    if (tid == 0) {
      const uint8_t* src;
      unsigned bytes;
      if (next_piece(p, cta, s.cur, &src, &bytes)) {
        issue_piece(s.ring + (size_t)slot * p.slot_bytes, src, bytes, s.full + slot);
        ++s.issued;
      }
    }
    ++s.consumed;
    const int row0 = pu0 * U;
    for (int r = tid; r < rows; r += nth) {
      const float* pr = s.part + r * rstride;
      float acc = 0.0f;
      for (int i = 0; i < nb; ++i) acc = __fadd_rn(acc, pr[i]);
      const float v = __fmul_rn(acc, act_scale);
      if (EPI == LE_ADD) {
        const int rg = row0 + r;
        const float nx = __fadd_rn(__ldcg(p.x + rg), v);
        __stcg(p.x + rg, nx);
        if (trace) trace[(size_t)(layer + 1) * p.n_embd + rg] = nx;
      } else {
        s.vals[r] = v;
      }
    }
    if (EPI != LE_ADD) __syncthreads();
    if (EPI == LE_QKV) {
      const int P = *p.pos;
      const LoopLayer& L = p.layers[layer];
      for (int r = tid; r < rows; r += nth) {
        const int rg = row0 + r;
        const float mine = s.vals[r];
        if (rg < p.nq + p.nkv) {
          const float other = s.vals[r ^ 1];
          const int rr = rg < p.nq ? rg : rg - p.nq;
          const int i = (rr % p.hd) >> 1;
          const float c = p.rope_cos[(size_t)P * (p.hd >> 1) + i];
          const float sn = p.rope_sin[(size_t)P * (p.hd >> 1) + i];
          const bool odd = r & 1;
          const float x0 = odd ? other : mine, x1 = odd ? mine : other;
          const float o = odd ? __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c))
                              : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
          if (rg < p.nq) {
            __stcg(p.q + rg, o);
          } else {
            const size_t idx = ((size_t)(rr / p.hd) * p.n_ctx + P) * p.hd + rr % p.hd;
            if (p.kv_f16) reinterpret_cast<__half*>(L.kc)[idx] = __float2half_rn(o);
            else reinterpret_cast<float*>(L.kc)[idx] = o;
          }
        } else {
          const int rr = rg - p.nq - p.nkv;
          const size_t idx = ((size_t)(rr / p.hd) * p.n_ctx + P) * p.hd + rr % p.hd;
          if (p.kv_f16) reinterpret_cast<__half*>(L.vc)[idx] = __float2half_rn(mine);
          else reinterpret_cast<float*>(L.vc)[idx] = mine;
        }
      }
    }
    if (EPI == LE_SWIGLU) {
      const int hu = U >> 1;
      for (int q = tid; q < pn * hu; q += nth) {
        const int ul = q / hu, i = q - ul * hu;
        const float gt = s.vals[ul * U + i], up = s.vals[ul * U + hu + i];
        const float o = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf_cr(-gt))), up);
        __stcg(p.h + (size_t)(pu0 + ul) * hu + i, o);
        am = absmax_acc(am, o);
      }
    }
    __syncthreads();  // vals and part are reused by the next piece
  }
  if (EPI == LE_SWIGLU) {
    am = block_reduce<float>(am, s.red + 64, OpMax(), 0.0f);
    if (tid == 0) *am_out = am;
  }
  return true;
}

template <int DPL>
__global__ void __launch_bounds__(LOOP_THREADS, 1) loop_kernel(const LoopParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int flag_sh;
  const int tid = threadIdx.x, nth = blockDim.x, cta = blockIdx.x, G = gridDim.x;
  LoopState s;
  s.ring = smem + p.ring_off;
  s.full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  s.xq = reinterpret_cast<int8_t*>(smem + p.xq_off);
  s.part = reinterpret_cast<float*>(smem + p.part_off);
  s.vals = reinterpret_cast<float*>(smem + p.vals_off);
  s.scr = reinterpret_cast<float*>(smem + p.scr_off);
  s.red = reinterpret_cast<float*>(smem + p.red_off);
  s.flag = &flag_sh;
  s.consumed = 0;
  s.issued = 0;
  s.cur = PieceCursor{0, 0, 0};
  s.nbar = 0;
  // every CTA reads the barrier base before its first arrival
  s.base = *reinterpret_cast<volatile unsigned*>(p.bar + 1);
  if (tid == 0) {
    for (int k = 0; k < p.n_slots; ++k) mbar_init(s.full + k, 1);
    mbar_fence_init();
    for (int k = 0; k < p.n_slots; ++k) {
      const uint8_t* src;
      unsigned bytes;
      if (!next_piece(p, cta, s.cur, &src, &bytes)) break;
      issue_piece(s.ring + (size_t)k * p.slot_bytes, src, bytes, s.full + k);
      ++s.issued;
    }
  }
  __syncthreads();

  const int K4 = p.n_embd >> 2;
  const int P = *p.pos + 1;
  const int gqa = p.n_head / p.n_kv;
  TileArgs ta;
  ta.q = p.q; ta.out = p.att; ta.part = p.part; ta.cnt = p.cnt; ta.amax = p.amax_att;
  ta.f16 = p.kv_f16; ta.n_ctx = p.n_ctx; ta.hd = p.hd; ta.gqa = gqa; ta.nt = p.attn_nt; ta.P = P;
  ta.scale = p.attn_scale;
  const int T = attn_tile_len(P, p.attn_nt), n_tiles = (P + T - 1) / T;
  const int n_items = p.attn_exact ? p.n_head : p.n_kv * n_tiles;
  const int n_att_slots = p.attn_exact ? p.n_head : p.n_kv;
  // the attention's shared memory (aliases xq, part and vals, idle then):
  // scores, small scratch, then the staged K and V chunks
  const int T_max = attn_tile_len(p.n_ctx, p.attn_nt);
  float* a_sc = s.scr;
  float* a_sm = a_sc + (size_t)gqa * T_max;
  TileStage st;
  st.ch = p.attn_ch;
  st.k = reinterpret_cast<uint8_t*>(a_sm + attn_sm_floats(p.attn_nt, gqa));
  st.v = st.k + (size_t)st.ch * p.hd * (p.kv_f16 ? 2 : 4);

  // the embedding (upstream src/forward.c:259-293), computed by every CTA for
  // its first prologue; CTA 0 also stores it as the residual
  float4 xv[LOOP_MAX_KR], nwv[LOOP_MAX_KR];
  {
    const uint8_t* row = p.embd + (size_t)(*p.token) * p.embd_rb;
#pragma unroll
    for (int k = 0; k < LOOP_MAX_KR; ++k) {
      const int i4 = tid + k * nth;
      if (i4 < K4) {
        const int e = i4 * 4;
        xv[k] = make_float4(dequant_elem(p.embd_type, row, e), dequant_elem(p.embd_type, row, e + 1),
                            dequant_elem(p.embd_type, row, e + 2), dequant_elem(p.embd_type, row, e + 3));
        if (cta == 0) {
          __stcg(reinterpret_cast<float4*>(p.x) + i4, xv[k]);
          if (p.trace) reinterpret_cast<float4*>(p.trace)[i4] = xv[k];
        }
      }
    }
  }
  bool ok = true;
  for (int l = 0; l < p.n_layer && ok; ++l) {
    const LoopLayer& L = p.layers[l];
    // ---- q|k|v: RMSNorm + quantise, GEMV, RoPE, K/V write
#pragma unroll
    for (int k = 0; k < LOOP_MAX_KR; ++k) {
      const int i4 = tid + k * nth;
      if (i4 < K4) nwv[k] = __ldg(reinterpret_cast<const float4*>(L.attn_norm) + i4);
    }
    if (l > 0) {
      if (!(ok = loop_barrier(p, s))) break;  // down of the previous layer
#pragma unroll
      for (int k = 0; k < LOOP_MAX_KR; ++k) {
        const int i4 = tid + k * nth;
        if (i4 < K4) xv[k] = __ldcg(reinterpret_cast<const float4*>(p.x) + i4);
      }
    }
    float sc = pro_norm(p, s, xv, nwv, p.n_embd);
    if (!(ok = loop_gemv<LE_QKV>(p, s, L.m[LM_QKV], sc, l, nullptr, nullptr))) break;
    // the older K/V rows of this CTA's first tile move while the others finish
    ta.kc = L.kc;
    ta.vc = L.vc;
    if (!p.attn_exact && cta < n_items) attn_tile_stage0(ta, st, cta / n_tiles, cta % n_tiles);
    if (!(ok = loop_barrier(p, s))) break;
    // every CTA has read the base by now: the next launch starts after this
    // launch's 5 * n_layer - 1 barriers
    if (l == 0 && cta == 0 && tid == 0) p.bar[1] = s.base + (unsigned)((5 * p.n_layer - 1) * G);

    // ---- attention
    for (int it = cta; it < n_items; it += G) {
      if (p.attn_exact) {
        attn_exact_head(ta, it, s.scr, s.red + 64, s.red + 96);
      } else {
        const int g = it / n_tiles, t = it - g * n_tiles;
        if (it != cta) attn_tile_stage0(ta, st, g, t);
        attn_tile<DPL>(ta, st, g, t, a_sc, a_sm);
        __syncthreads();
        attn_merge_tiles(ta, g, a_sm, s.red + 64);
      }
      __syncthreads();
    }
    if (!(ok = loop_barrier(p, s))) break;

    // ---- o (+ residual)
    sc = pro_vec(s, p.att, p.nq, p.amax_att, n_att_slots);
    if (!(ok = loop_gemv<LE_ADD>(p, s, L.m[LM_O], sc, l, nullptr, nullptr))) break;
#pragma unroll
    for (int k = 0; k < LOOP_MAX_KR; ++k) {
      const int i4 = tid + k * nth;
      if (i4 < K4) nwv[k] = __ldg(reinterpret_cast<const float4*>(L.ffn_norm) + i4);
    }
    if (!(ok = loop_barrier(p, s))) break;

    // ---- gate|up: RMSNorm + quantise, GEMV, SwiGLU
#pragma unroll
    for (int k = 0; k < LOOP_MAX_KR; ++k) {
      const int i4 = tid + k * nth;
      if (i4 < K4) xv[k] = __ldcg(reinterpret_cast<const float4*>(p.x) + i4);
    }
    sc = pro_norm(p, s, xv, nwv, p.n_embd);
    {
      float h_am = 0.0f;
      if (!(ok = loop_gemv<LE_SWIGLU>(p, s, L.m[LM_GU], sc, l, nullptr, &h_am))) break;
      if (tid == 0) __stcg(p.amax_h + cta, h_am);
    }
    if (!(ok = loop_barrier(p, s))) break;

    // ---- down (+ residual)
    sc = pro_vec(s, p.h, p.n_ff, p.amax_h, G);
    if (!(ok = loop_gemv<LE_ADD>(p, s, L.m[LM_DOWN], sc, l, p.trace, nullptr))) break;
  }
  cp_async_wait_all();
  if (!ok) drain_copies(p, s);
}

}  // namespace fox
