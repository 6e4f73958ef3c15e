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
// after about a second (then the error word is set).
FOX_DEV bool grid_barrier(unsigned* bar, unsigned target, int* err, int* ok_sh) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    red_release_gpu_add(bar, 1u);
    int ok = 0;
    const uint64_t t0 = globaltimer_ns();
    for (int i = 0;; ++i) {
      if ((int)(ld_acquire_gpu(bar) - target) >= 0) { ok = 1; break; }
      if ((i & 63) == 63 && globaltimer_ns() - t0 > 1000000000ull) break;
      if (i > 64) __nanosleep(32);
    }
    if (!ok && err) atomicExch(err, 3);
    __threadfence();
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

// Tile t of KV group g: the partials of every query head of the group. The
// shared scratch holds gqa * T floats (scores, then weights) and 4 * 32 more.
template <int DPL>
FOX_DEV void attn_tile(const TileArgs& a, int g, int t, float* sc, float* sm) {
  const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nth >> 5;
  const int T = attn_tile_len(a.P, a.nt);
  const int j0 = t * T, n = min(T, a.P - j0);
  const int hd = a.hd, gqa = a.gqa;
  const bool f16 = a.f16 != 0;
  const size_t head = (size_t)g * a.n_ctx * hd;
  float qv[LOOP_MAX_GQA][DPL];
#pragma unroll
  for (int h = 0; h < LOOP_MAX_GQA; ++h)
#pragma unroll
    for (int i = 0; i < DPL; ++i)
      qv[h][i] = h < gqa ? __ldcg(a.q + ((size_t)g * gqa + h) * hd + lane * DPL + i) : 0.0f;
  for (int j = warp; j < n; j += nw) {
    float k[DPL];
    load_row<DPL>(a.kc, f16, head + (size_t)(j0 + j) * hd + lane * DPL, k);
#pragma unroll
    for (int h = 0; h < LOOP_MAX_GQA; ++h) {
      if (h >= gqa) break;
      float d = __fmul_rn(qv[h][0], k[0]);
#pragma unroll
      for (int i = 1; i < DPL; ++i) d = __fmaf_rn(qv[h][i], k[i], d);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, o));
      if (lane == 0) sc[h * T + j] = __fmul_rn(d, a.scale);
    }
  }
  __syncthreads();
  float* s_m = sm;          // [gqa]
  float* s_l = sm + 32;     // [gqa]
  if (warp < gqa) {
    float mx = -CUDART_INF_F;
    for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[warp * T + j]);
    mx = warp_max(mx);
    if (lane == 0) s_m[warp] = mx;
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
  float* part = a.part + ((size_t)g * a.nt + t) * gqa * (hd + 2);
  // one thread per dimension holds every head's sum: each V element is read once
  for (int d = tid; d < hd; d += nth) {
    float o[LOOP_MAX_GQA];
#pragma unroll
    for (int h = 0; h < LOOP_MAX_GQA; ++h) o[h] = 0.0f;
#pragma unroll 4
    for (int j = 0; j < n; ++j) {
      const float v = load_elem(a.vc, f16, head + (size_t)(j0 + j) * hd + d);
#pragma unroll
      for (int h = 0; h < LOOP_MAX_GQA; ++h)
        if (h < gqa) o[h] = __fmaf_rn(sc[h * T + j], v, o[h]);
    }
#pragma unroll
    for (int h = 0; h < LOOP_MAX_GQA; ++h)
      if (h < gqa) __stcg(part + (size_t)h * (hd + 2) + d, o[h]);
  }
  __syncthreads();
  if (tid < gqa) {
    __stcg(part + (size_t)tid * (hd + 2) + hd, s_m[tid]);
    __stcg(part + (size_t)tid * (hd + 2) + hd + 1, s_l[tid]);
  }
}

// After attn_tile: the CTA that completes KV group g's last tile merges all
// its tiles into the output (and publishes the absmax of what it wrote).
// The scratch holds 3 * nt * gqa + 2 * gqa floats.
FOX_DEV void attn_merge_tiles(const TileArgs& a, int g, float* sm, float* red) {
  __shared__ int last_sh;
  const int tid = threadIdx.x, nth = blockDim.x;
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
  for (int i = tid; i < nt * gqa; i += nth) {
    const float* pt = base + (size_t)i * (hd + 2);
    s_m[i] = __ldcg(pt + hd);
    s_l[i] = __ldcg(pt + hd + 1);
  }
  __syncthreads();
  if (tid < gqa) {
    float M = -CUDART_INF_F;
    for (int t = 0; t < nt; ++t) M = fmaxf(M, s_m[t * gqa + tid]);
    s_M[tid] = M;
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
    for (int t = 0; t < nt; ++t)
      O = __fmaf_rn(__ldcg(base + ((size_t)t * gqa + h) * (hd + 2) + d), s_w[t * gqa + h], O);
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
// kcache / vcache), and uses the partials and counters of slot z.
template <int DPL>
__global__ void __launch_bounds__(256, 1) attention_tile_kernel(const AttnParams k) {
  extern __shared__ __align__(16) float tsm[];
  __shared__ float red[32];
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
  float* sc = tsm;                       // gqa * T
  float* sm = tsm + (size_t)gqa * T;     // max(64, 3 * nt * gqa + 2 * gqa)
  attn_tile<DPL>(a, g, t, sc, sm);
  attn_merge_tiles(a, g, sm, red);
}

// Shared memory of attention_tile_kernel for contexts of n_ctx positions.
inline size_t attn_tile_smem_bytes(int n_ctx, int nt, int gqa) {
  const int T = attn_tile_len(n_ctx, nt);
  return ((size_t)gqa * T + (size_t)std::max(64, 3 * nt * gqa + 2 * gqa)) * 4;
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
    if (!(ok = loop_barrier(p, s))) break;
    // every CTA has read the base by now: the next launch starts after this
    // launch's 5 * n_layer - 1 barriers
    if (l == 0 && cta == 0 && tid == 0) p.bar[1] = s.base + (unsigned)((5 * p.n_layer - 1) * G);

    // ---- attention
    ta.kc = L.kc;
    ta.vc = L.vc;
    for (int it = cta; it < n_items; it += G) {
      if (p.attn_exact) {
        attn_exact_head(ta, it, s.scr, s.red + 64, s.red + 96);
      } else {
        const int g = it / n_tiles, t = it - g * n_tiles;
        float* sm = s.scr + (size_t)gqa * T;
        attn_tile<DPL>(ta, g, t, s.scr, sm);
        attn_merge_tiles(ta, g, sm, s.red + 64);
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
  if (!ok) drain_copies(p, s);
}

}  // namespace fox
