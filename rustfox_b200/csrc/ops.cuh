// Non-GEMV device ops of the token loop: row dequantisation (embedding
// gather), split-K GQA decode attention over the K/V cache, and the sampler.
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace fox {

// ---------------------------------------------------------------------------
// Element e of a row in GGUF layout, as upstream's fox_dequant_row computes it
// (src/kernels.c:874-941; Q4_K src/kernels.c:257-283; Q6_K :217-244).
FOX_DEV float dequant_elem(int type, const uint8_t* row, int e) {
  switch (type) {
    case T_F32: return reinterpret_cast<const float*>(row)[e];
    case T_F16: return h2f((uint16_t)(row[2 * e] | (row[2 * e + 1] << 8)));
    case T_Q8_0: {
      const uint8_t* b = row + (e >> 5) * 34;
      const float d = h2f((uint16_t)(b[0] | (b[1] << 8)));
      return __fmul_rn((float)(int8_t)b[2 + (e & 31)], d);
    }
    case T_Q4_K: {
      const uint8_t* b = row + (e >> 8) * 144;
      const int i = e & 255, j = i >> 5, l = i & 31;
      const float d = h2f((uint16_t)(b[0] | (b[1] << 8)));
      const float dmin = h2f((uint16_t)(b[2] | (b[3] << 8)));
      const uint8_t* s = b + 4;
      int sc, m;
      if (j < 4) { sc = s[j] & 63; m = s[j + 4] & 63; }
      else { sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4); m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
      const uint8_t q = b[16 + (j >> 1) * 32 + l];
      const int nib = (j & 1) ? (q >> 4) : (q & 0x0F);
      return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)nib), __fmul_rn(dmin, (float)m));
    }
    case T_Q6_K: {
      const uint8_t* b = row + (e >> 8) * 210;
      const int i = e & 255, half = i >> 7, g = (i & 127) >> 5, l = i & 31;
      const uint8_t* ql = b + half * 64;
      const uint8_t* qh = b + 128 + half * 32;
      const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192) + half * 8;
      int lo = (g & 1) ? ql[l + 32] : ql[l];
      lo = (g & 2) ? (lo >> 4) : (lo & 0x0F);
      const int q = (lo | (((qh[l] >> (2 * g)) & 3) << 4)) - 32;
      const float d = h2f((uint16_t)(b[208] | (b[209] << 8)));
      return __fmul_rn(__fmul_rn(d, (float)sc[(l >> 4) + 2 * g]), (float)q);
    }
    default: return 0.0f;
  }
}

__global__ void dequant_row_kernel(int type, const uint8_t* __restrict__ row, int n,
                                   float* __restrict__ out) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x)
    out[e] = dequant_elem(type, row, e);
}

// Embedding row of the token held in device memory (upstream src/forward.c:259-293).
__global__ void embed_kernel(int type, const uint8_t* __restrict__ table, size_t row_bytes,
                             int n_embd, const uint32_t* __restrict__ token,
                             float* __restrict__ x) {
  griddep_launch_dependents();  // the first q|k|v GEMV may start streaming its weights
  const uint8_t* row = table + (size_t)(*token) * row_bytes;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n_embd; e += gridDim.x * blockDim.x)
    x[e] = dequant_elem(type, row, e);
}

// The same, for a token given as a launch argument (kept in *token for the
// next step): nothing in host memory is read after the launch.
__global__ void embed_token_kernel(int type, const uint8_t* __restrict__ table, size_t row_bytes,
                                   int n_embd, uint32_t tok, uint32_t* token,
                                   float* __restrict__ x) {
  if (blockIdx.x == 0 && threadIdx.x == 0) *token = tok;
  const uint8_t* row = table + (size_t)tok * row_bytes;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n_embd; e += gridDim.x * blockDim.x)
    x[e] = dequant_elem(type, row, e);
}

__global__ void advance_kernel(int* pos, int by) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *pos += by;
}

// ---------------------------------------------------------------------------
// Decode attention (upstream src/forward.c:222-257 + src/ops.c:24-39,75-81):
// per query head, scores q.k_j * (1/sqrtf(hd)) for j <= pos, softmax, sum of
// a_j v_j. Flash-decoding form: CTA (s, g) takes split s of the positions for
// KV head g and all its query heads (the K/V rows are read once per group),
// keeps an online softmax per warp, and writes (max, sum, unnormalised
// output) partials; the last CTA of a KV head to finish merges them.

struct AttnParams {
  const float* q;         // [n_head * hd], roped
  const void* kcache;     // this layer: [n_kv][n_ctx][hd]
  const void* vcache;
  int kv_f16, n_ctx, hd, n_head, n_kv, S_max;
  const int* pos;
  float* out;             // [n_head * hd]
  float* part;            // [n_kv][S_max][gqa][hd + 2]
  unsigned* counters;     // [n_kv], zero between launches
  float scale;
  // 1: launched with programmatic stream serialisation right after the
  // kernel that wrote q and position *pos of the cache; rows before *pos
  // were written by earlier launches and are staged before the wait
  int pdl;
  // decode batches (attention_cluster_kernel<..., SEQS>): sequence z reads
  // q + z * seq_stride, writes out + z * seq_stride, its position at
  // *pos_list[z] and its layer's caches at k_list[z] / v_list[z] + layer_off
  int seq_stride;
  int* const* pos_list;
  void* const* k_list;
  void* const* v_list;
  size_t layer_off;
};

constexpr int ATTN_THREADS = 128;
constexpr int ATTN_MAX_GQA = 8;
constexpr int ATTN_MAX_DPL = 8;  // head_dim <= 256

template <int DPL>
FOX_DEV void load_kv(const void* cache, bool f16, size_t off, float* v) {
  if (f16) {
    const __half* p = reinterpret_cast<const __half*>(cache) + off;
    if (DPL == 4) {
      const uint2 r = *reinterpret_cast<const uint2*>(p);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
#pragma unroll
      for (int i = 0; i < DPL; ++i) v[i] = __half2float(p[i]);
    }
  } else {
    const float* p = reinterpret_cast<const float*>(cache) + off;
#pragma unroll
    for (int i = 0; i < DPL; ++i) v[i] = p[i];
  }
}

// The last CTA of KV head g to finish merges the S split partials
// (max, sum, unnormalised output per query head) into the output.
FOX_DEV void attn_merge(const AttnParams& p, int g, int S, int gqa, int hd) {
  __shared__ bool is_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(p.counters + g, 1u) == (unsigned)(S - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // The partials of the other CTAs are read through L2 (ld.global.cg: L1 is
  // not coherent with their writes). Per (split, head): max and sum to shared
  // memory, then the rescale factors, then every output dimension as an
  // independent, pipelined sweep over the splits.
  __shared__ float s_m[32][ATTN_MAX_GQA], s_l[32][ATTN_MAX_GQA], s_e[32][ATTN_MAX_GQA];
  __shared__ float s_M[ATTN_MAX_GQA], s_L[ATTN_MAX_GQA];
  const float* base = p.part + (size_t)g * p.S_max * gqa * (hd + 2);
  for (int i = threadIdx.x; i < S * gqa; i += blockDim.x) {
    const int t = i / gqa, h = i % gqa;
    const float* pt = base + ((size_t)t * gqa + h) * (hd + 2);
    s_m[t][h] = __ldcg(pt + hd);
    s_l[t][h] = __ldcg(pt + hd + 1);
  }
  __syncthreads();
  if (threadIdx.x < gqa) {
    const int h = threadIdx.x;
    float M = -CUDART_INF_F;
    for (int t = 0; t < S; ++t)
      if (s_l[t][h] > 0.0f) M = fmaxf(M, s_m[t][h]);
    s_M[h] = M;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < S * gqa; i += blockDim.x) {
    const int t = i / gqa, h = i % gqa;
    s_e[t][h] = s_l[t][h] > 0.0f ? expf_cr(s_m[t][h] - s_M[h]) : 0.0f;
  }
  __syncthreads();
  if (threadIdx.x < gqa) {
    const int h = threadIdx.x;
    float L = 0.0f;
    for (int t = 0; t < S; ++t)
      if (s_l[t][h] > 0.0f) L = fmaf(s_l[t][h], s_e[t][h], L);
    s_L[h] = L;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < gqa * hd; idx += blockDim.x) {
    const int h = idx / hd, d = idx % hd;
    float A = 0.0f;
#pragma unroll 8
    for (int t = 0; t < S; ++t) {
      const float v = __ldcg(base + ((size_t)t * gqa + h) * (hd + 2) + d);
      if (s_l[t][h] > 0.0f) A = fmaf(v, s_e[t][h], A);
    }
    p.out[(g * gqa + h) * hd + d] = A / s_L[h];
  }
  if (threadIdx.x == 0) p.counters[g] = 0u;
}

template <int DPL>
__global__ void __launch_bounds__(ATTN_THREADS) attention_kernel(const AttnParams p) {
  griddep_launch_dependents();  // the o projection may start streaming its weights
  const int s = blockIdx.x, g = blockIdx.y;
  const int P = *p.pos + 1;
  const int S = min(p.S_max, max(1, (P + 31) / 32));
  if (s >= S) return;
  const int chunk = (P + S - 1) / S;
  const int j0 = s * chunk, j1 = min(P, j0 + chunk);
  const int gqa = p.n_head / p.n_kv, hd = p.hd;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool f16 = p.kv_f16 != 0;

  __shared__ float qs[ATTN_MAX_GQA * 32 * ATTN_MAX_DPL];
  __shared__ float wm[4][ATTN_MAX_GQA], wl[4][ATTN_MAX_GQA];
  __shared__ float wacc[4][ATTN_MAX_GQA * 32 * ATTN_MAX_DPL];

  for (int i = threadIdx.x; i < gqa * hd; i += blockDim.x) qs[i] = p.q[g * gqa * hd + i];
  __syncthreads();

  float m[ATTN_MAX_GQA], l[ATTN_MAX_GQA], acc[ATTN_MAX_GQA][DPL];
#pragma unroll
  for (int h = 0; h < ATTN_MAX_GQA; ++h) {
    m[h] = -CUDART_INF_F; l[h] = 0.0f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[h][i] = 0.0f;
  }
  const size_t head_base = (size_t)g * p.n_ctx * hd + lane * DPL;
  for (int j = j0 + warp; j < j1; j += 4) {
    float k[DPL], v[DPL];
    load_kv<DPL>(p.kcache, f16, head_base + (size_t)j * hd, k);
    load_kv<DPL>(p.vcache, f16, head_base + (size_t)j * hd, v);
#pragma unroll
    for (int h = 0; h < ATTN_MAX_GQA; ++h) {
      if (h >= gqa) continue;
      float d = 0.0f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) d = fmaf(qs[h * hd + lane * DPL + i], k[i], d);
      const float sc = warp_sum(d) * p.scale;
      const float mn = fmaxf(m[h], sc);
      const float corr = expf_cr(m[h] - mn);
      const float pr = expf_cr(sc - mn);
      l[h] = l[h] * corr + pr;
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[h][i] = fmaf(pr, v[i], acc[h][i] * corr);
      m[h] = mn;
    }
  }
  // merge the four warps
#pragma unroll
  for (int h = 0; h < ATTN_MAX_GQA; ++h) {
    if (h >= gqa) continue;
    if (lane == 0) { wm[warp][h] = m[h]; wl[warp][h] = l[h]; }
#pragma unroll
    for (int i = 0; i < DPL; ++i) wacc[warp][h * hd + lane * DPL + i] = acc[h][i];
  }
  __syncthreads();
  float* part = p.part + ((size_t)g * p.S_max + s) * gqa * (hd + 2);
  for (int idx = threadIdx.x; idx < gqa * hd; idx += blockDim.x) {
    const int h = idx / hd;
    float M = -CUDART_INF_F;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][h]);
    float A = 0.0f, L = 0.0f;
    for (int w = 0; w < 4; ++w) {
      const float e = wl[w][h] > 0.0f ? expf_cr(wm[w][h] - M) : 0.0f;
      A = fmaf(wacc[w][idx], e, A);
      L = fmaf(wl[w][h], e, L);
    }
    part[h * (hd + 2) + idx % hd] = A;
    if (idx % hd == 0) { part[h * (hd + 2) + hd] = M; part[h * (hd + 2) + hd + 1] = L; }
  }
  attn_merge(p, g, S, gqa, hd);
}

// Shared memory of one attention tile: 128 K rows padded by 16 bytes, then
// 128 V rows.
template <int HD, bool F16>
constexpr size_t attn_tile_smem() {
  return (size_t)128 * (HD * (F16 ? 2 : 4) + 16) + (size_t)128 * HD * (F16 ? 2 : 4);
}

FOX_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
FOX_DEV void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
}

// Cluster decode attention. The ATTN_SPLITS CTAs of one KV head form a
// thread-block cluster; CTA r takes the r-th run of the positions, in tiles of
// 128 (K/V staged in shared memory with cp.async before q is read, scores one
// position per thread, a per-tile online softmax, the weighted V sum one
// dimension per thread). Its partial (max, sum, unnormalised output per query
// head) stays in its own shared memory. After a cluster barrier every CTA
// merges 1/ATTN_SPLITS of the outputs by reading the others' partials through
// distributed shared memory, and a second barrier keeps every partial alive
// until the last remote read. No global scratch, fence or atomic.
constexpr int ATTN_SPLITS = 8;  // portable cluster size

FOX_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// address of the same shared variable in CTA `rank` of this cluster
FOX_DEV const float* cluster_peer(const float* p, unsigned rank) {
  uint64_t r;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(p), "r"(rank));
  return reinterpret_cast<const float*>(r);
}

// SEQS: one launch for a decode batch; grid z is the sequence, whose q, out,
// position and caches come from AttnParams' per-sequence fields.
template <int HD, int G, bool F16, bool SEQS = false>
__global__ void __cluster_dims__(ATTN_SPLITS, 1, 1) __launch_bounds__(128)
attention_cluster_kernel(const AttnParams p) {
  griddep_launch_dependents();  // the o projection may start streaming its weights
  constexpr int NT = 128, DPT = NT / HD;
  constexpr int ESZ = F16 ? 2 : 4, RB = HD * ESZ, KSTRIDE = RB + 16;
  const int r = blockIdx.x, g = blockIdx.y, tid = threadIdx.x;  // r = rank in the cluster
  const int lane = tid & 31, warp = tid >> 5;
  const float* q_in = p.q;
  float* out = p.out;
  const int* pos = p.pos;
  const void* kcache = p.kcache;
  const void* vcache = p.vcache;
  if constexpr (SEQS) {
    const int z = blockIdx.z;
    q_in = p.q + (size_t)z * p.seq_stride;
    out = p.out + (size_t)z * p.seq_stride;
    pos = p.pos_list[z];
    kcache = reinterpret_cast<const uint8_t*>(p.k_list[z]) + p.layer_off;
    vcache = reinterpret_cast<const uint8_t*>(p.v_list[z]) + p.layer_off;
  }
  const int P = *pos + 1;
  const int chunk = (P + ATTN_SPLITS - 1) / ATTN_SPLITS;
  const int j0 = min(P, r * chunk), j1 = min(P, j0 + chunk);

  extern __shared__ __align__(16) unsigned char smem[];
  uint8_t* sK = smem;
  uint8_t* sV = smem + (size_t)NT * KSTRIDE;
  __shared__ float qs[G][HD];
  __shared__ float ps[G][NT];
  __shared__ float rmax[4][G], rsum[4][G];
  __shared__ float accs[DPT > 1 ? DPT - 1 : 1][G][HD];
  __shared__ float part[G][HD + 2];           // this CTA's partial, read by the cluster
  __shared__ float ew[ATTN_SPLITS][G], lw[ATTN_SPLITS][G];

  const size_t head = (size_t)g * p.n_ctx * HD;
  const uint8_t* kg = reinterpret_cast<const uint8_t*>(kcache) + head * ESZ;
  const uint8_t* vg = reinterpret_cast<const uint8_t*>(vcache) + head * ESZ;
  // rows t0 .. t0+n-1 of the cache into tile rows 0 .. n-1, except position skip
  auto stage = [&](int t0, int n, int skip) {
    const int pieces = n * (RB / 16);
    for (int i = tid; i < pieces; i += NT) {
      const int row = i / (RB / 16), c = i - row * (RB / 16);
      if (t0 + row == skip) continue;
      cp_async16(sK + (size_t)row * KSTRIDE + c * 16, kg + (size_t)(t0 + row) * RB + c * 16);
      cp_async16(sV + (size_t)i * 16, vg + (size_t)t0 * RB + (size_t)i * 16);
    }
  };
  // The first tile is in flight while q is read. Under programmatic launch
  // the newest position (P - 1) and q come from the kernel still finishing:
  // they are read after griddepcontrol.wait (a no-op for a plain launch).
  const int n0 = j0 < j1 ? min(NT, j1 - j0) : 0;
  const int cur = p.pdl ? P - 1 : -1;
  if (n0) stage(j0, n0, cur);
  griddep_wait();
  if (cur >= j0 && cur < j0 + n0)
    for (int c = tid; c < RB / 16; c += NT) {
      const int row = cur - j0;
      cp_async16(sK + (size_t)row * KSTRIDE + c * 16, kg + (size_t)cur * RB + c * 16);
      cp_async16(sV + (size_t)row * RB + c * 16, vg + (size_t)cur * RB + c * 16);
    }
  for (int i = tid; i < G * HD; i += NT) qs[i / HD][i % HD] = q_in[(size_t)g * G * HD + i];

  const int d = tid % HD, jsub = tid / HD;
  float m[G], l[G], acc[G];
#pragma unroll
  for (int h = 0; h < G; ++h) { m[h] = -CUDART_INF_F; l[h] = 0.0f; acc[h] = 0.0f; }

  for (int t0 = j0; t0 < j1; t0 += NT) {
    const int n = min(NT, j1 - t0);
    if (t0 != j0) stage(t0, n, -1);
    cp_async_wait_all();
    __syncthreads();
    const bool on = tid < n;
    float sc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) sc[h] = 0.0f;
    if (on) {
      const uint4* kr = reinterpret_cast<const uint4*>(sK + (size_t)tid * KSTRIDE);
#pragma unroll 4
      for (int c = 0; c < RB / 16; ++c) {
        const uint4 w = kr[c];
        if (F16) {
          const __half2* hw = reinterpret_cast<const __half2*>(&w);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 kv = __half22float2(hw[e]);
#pragma unroll
            for (int h = 0; h < G; ++h) {
              sc[h] = fmaf(qs[h][c * 8 + 2 * e], kv.x, sc[h]);
              sc[h] = fmaf(qs[h][c * 8 + 2 * e + 1], kv.y, sc[h]);
            }
          }
        } else {
          const float* fw = reinterpret_cast<const float*>(&w);
#pragma unroll
          for (int e = 0; e < 4; ++e)
#pragma unroll
            for (int h = 0; h < G; ++h) sc[h] = fmaf(qs[h][c * 4 + e], fw[e], sc[h]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      sc[h] = on ? sc[h] * p.scale : -CUDART_INF_F;
      const float mx = warp_max(sc[h]);
      if (lane == 0) rmax[warp][h] = mx;
    }
    __syncthreads();
    float corr[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float tmax = fmaxf(fmaxf(rmax[0][h], rmax[1][h]), fmaxf(rmax[2][h], rmax[3][h]));
      const float mn = fmaxf(m[h], tmax);
      corr[h] = m[h] == -CUDART_INF_F ? 0.0f : expf_cr(m[h] - mn);
      float pj = 0.0f;
      if (on) pj = expf_cr(sc[h] - mn);
      ps[h][tid] = pj;
      const float sm = warp_sum(pj);
      if (lane == 0) rsum[warp][h] = sm;
      m[h] = mn;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < G; ++h) {
      l[h] = fmaf(l[h], corr[h], (rsum[0][h] + rsum[1][h]) + (rsum[2][h] + rsum[3][h]));
      acc[h] *= corr[h];
    }
#pragma unroll 8
    for (int jj = jsub; jj < n; jj += DPT) {
      const float v = F16 ? __half2float(reinterpret_cast<const __half*>(sV)[(size_t)jj * HD + d])
                          : reinterpret_cast<const float*>(sV)[(size_t)jj * HD + d];
#pragma unroll
      for (int h = 0; h < G; ++h) acc[h] = fmaf(ps[h][jj], v, acc[h]);
    }
    __syncthreads();
  }
  if (DPT > 1) {
    if (jsub > 0)
#pragma unroll
      for (int h = 0; h < G; ++h) accs[jsub - 1][h][d] = acc[h];
    __syncthreads();
    if (jsub == 0)
#pragma unroll
      for (int h = 0; h < G; ++h)
        for (int k = 0; k < DPT - 1; ++k) acc[h] += accs[k][h][d];
  }
  if (jsub == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      part[h][d] = acc[h];
      if (d == 0) { part[h][HD] = m[h]; part[h][HD + 1] = l[h]; }
    }
  }
  cluster_sync_all();
  // merge: rescale factors of every split, then this CTA's slice of outputs
  if (tid < ATTN_SPLITS * G) {
    const int t = tid / G, h = tid - t * G;
    const float* pt = cluster_peer(&part[h][0], t);
    ew[t][h] = pt[HD];
    lw[t][h] = pt[HD + 1];
  }
  __syncthreads();
  if (tid < G) {
    const int h = tid;
    float M = -CUDART_INF_F;
    for (int t = 0; t < ATTN_SPLITS; ++t)
      if (lw[t][h] > 0.0f) M = fmaxf(M, ew[t][h]);
    float L = 0.0f;
    for (int t = 0; t < ATTN_SPLITS; ++t) {
      const float e = lw[t][h] > 0.0f ? expf_cr(ew[t][h] - M) : 0.0f;
      ew[t][h] = e;
      L = fmaf(lw[t][h], e, L);
    }
    rsum[0][h] = L;
  }
  __syncthreads();
  constexpr int PER = G * HD / ATTN_SPLITS;  // outputs merged by each CTA
  for (int k = tid; k < PER; k += NT) {
    const int idx = r * PER + k, h = idx / HD, dd = idx - h * HD;
    float A = 0.0f;
#pragma unroll
    for (int t = 0; t < ATTN_SPLITS; ++t)
      if (lw[t][h] > 0.0f) A = fmaf(cluster_peer(&part[h][dd], t)[0], ew[t][h], A);
    out[((size_t)g * G + h) * HD + dd] = A / rsum[0][h];
  }
  cluster_sync_all();  // no CTA leaves while another may still read its partial
}

// Attention in upstream's exact operation order (src/forward.c:222-257,
// src/ops.c:24-39,75-81), one CTA per query head: sequential dot products,
// scale, max, exp, a sequential sum, one reciprocal, and for each output
// dimension a sequential sum over positions. Slow (the sums are serial) but
// bit-identical to upstream given the same K/V and exp; the parity mode.
__global__ void attention_exact_kernel(const AttnParams p) {
  extern __shared__ float att[];  // positions 0..pos
  __shared__ float red[32];
  __shared__ float s_inv;
  __shared__ int s_pos;
  const int h = blockIdx.x, hd = p.hd, gqa = p.n_head / p.n_kv, kvh = h / gqa;
  const int P = *p.pos + 1;
  const float* qh = p.q + (size_t)h * hd;
  const size_t base = (size_t)kvh * p.n_ctx * hd;
  for (int j = threadIdx.x; j < P; j += blockDim.x) {
    float s = 0.0f;
    for (int d = 0; d < hd; ++d) {
      const size_t at = base + (size_t)j * hd + d;
      const float k = p.kv_f16 ? __half2float(reinterpret_cast<const __half*>(p.kcache)[at])
                               : reinterpret_cast<const float*>(p.kcache)[at];
      s = __fadd_rn(s, __fmul_rn(qh[d], k));
    }
    att[j] = __fmul_rn(s, p.scale);
  }
  __syncthreads();
  float mx = -CUDART_INF_F;
  for (int j = threadIdx.x; j < P; j += blockDim.x) mx = fmaxf(mx, att[j]);
  mx = block_reduce<float>(mx, red, OpMax(), -CUDART_INF_F);
  for (int j = threadIdx.x; j < P; j += blockDim.x) att[j] = expf_cr(__fsub_rn(att[j], mx));
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = 0.0f;
    for (int j = 0; j < P; ++j) sum = __fadd_rn(sum, att[j]);
    s_inv = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 0.0f;
    s_pos = sum > 0.0f;
  }
  __syncthreads();
  if (s_pos)
    for (int j = threadIdx.x; j < P; j += blockDim.x) att[j] = __fmul_rn(att[j], s_inv);
  __syncthreads();
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < P; ++j) {
      const size_t at = base + (size_t)j * hd + d;
      const float v = p.kv_f16 ? __half2float(reinterpret_cast<const __half*>(p.vcache)[at])
                               : reinterpret_cast<const float*>(p.vcache)[at];
      acc = __fadd_rn(acc, __fmul_rn(att[j], v));
    }
    p.out[(size_t)h * hd + d] = acc;
  }
}

// ---------------------------------------------------------------------------
// Sampler (upstream src/sample.c). State lives on the device so a captured
// decode step can pick and accept without the host.

constexpr int SAMPLER_MAX_HIST = 1024;
constexpr int ARGMAX_THREADS = 512;

struct SamplerDev {
  uint32_t hist[SAMPLER_MAX_HIST];
  float saved[SAMPLER_MAX_HIST];
  uint32_t hist_len, hist_head, hist_cap, pad0;
  unsigned long long rng;
  unsigned counter, pad1;
  float part_val[1024];
  uint32_t part_idx[1024];
  uint32_t token;          // last pick
  uint32_t n_out;          // picks written to the output ring so far
};

// Repeat penalty over the accepted history, in place on the logits; the
// original values are kept to be restored after the pick (src/sample.c:95-107:
// a token seen c times is divided or multiplied c times).
__global__ void penalty_kernel(SamplerDev* st, float* logits, int n_vocab, float penalty) {
  const int n = st->hist_len;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t tok = st->hist[i];
    bool first = tok < (uint32_t)n_vocab;
    for (int j = 0; j < i && first; ++j) first = st->hist[j] != tok;
    if (!first) continue;
    int c = 0;
    for (int j = 0; j < n; ++j) c += st->hist[j] == tok;
    float v = logits[tok];
    st->saved[i] = v;
    for (int r = 0; r < c; ++r) v = v > 0.0f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
    logits[tok] = v;
  }
}

FOX_DEV bool better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

FOX_DEV void accept_token(SamplerDev* st, uint32_t tok) {
  st->hist[st->hist_head] = tok;
  st->hist_head = (st->hist_head + 1) % st->hist_cap;
  if (st->hist_len < st->hist_cap) st->hist_len++;
}

// First strict maximum (ties to the lowest index, src/sample.c:147-153).
// The last CTA restores penalised logits, optionally accepts the pick into the
// history and publishes it (next-token slot and an output ring).
__global__ void __launch_bounds__(ARGMAX_THREADS)
argmax_kernel(SamplerDev* st, float* logits, int n_vocab, int restore, int accept,
              uint32_t* token_out, uint32_t* ring, int ring_cap) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  __shared__ bool is_last;
  float bv = -CUDART_INF_F;
  uint32_t bi = 0xffffffffu;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_vocab; i += gridDim.x * blockDim.x) {
    const float v = logits[i];
    if (better(v, i, bv, bi)) { bv = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
    st->part_val[blockIdx.x] = bv;
    st->part_idx[blockIdx.x] = bi;
    __threadfence();
    is_last = atomicAdd(&st->counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // merge the per-CTA winners in parallel, read through L2 (ld.global.cg)
  bv = -CUDART_INF_F;
  bi = 0xffffffffu;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) {
    const float v = __ldcg(st->part_val + b);
    const uint32_t i = __ldcg(st->part_idx + b);
    if (better(v, i, bv, bi)) { bv = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
    if (bi >= (uint32_t)n_vocab) bi = 0;  // all NaN: upstream keeps index 0
    st->counter = 0;
    st->token = bi;
    if (token_out) *token_out = bi;
    if (ring) { ring[st->n_out % ring_cap] = bi; st->n_out++; }
  }
  __syncthreads();
  if (restore) {
    const int n = st->hist_len;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t tok = st->hist[i];
      bool first = tok < (uint32_t)n_vocab;
      for (int j = 0; j < i && first; ++j) first = st->hist[j] != tok;
      if (first) logits[tok] = st->saved[i];
    }
  }
  __syncthreads();
  if (accept && threadIdx.x == 0) accept_token(st, st->token);
}

__global__ void accept_kernel(SamplerDev* st, uint32_t tok) {
  if (threadIdx.x == 0 && blockIdx.x == 0) accept_token(st, tok);
}

// Top-k / temperature / top-p draw (src/sample.c:155-194) in one CTA: radix
// select of the k-th largest (logit, lowest index first), a bitonic sort of
// the k candidates, then the upstream float sequence on one thread.
constexpr int TOPK_THREADS = 1024;
constexpr int TOPK_MAX = 512;

FOX_DEV uint32_t order_key(float f) {  // larger float -> larger key
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(TOPK_THREADS)
topk_sample_kernel(SamplerDev* st, float* logits, int n_vocab, int k, float temperature,
                   float top_p, int restore, int accept, uint32_t* token_out,
                   uint32_t* ring, int ring_cap) {
  __shared__ unsigned hist[256];
  __shared__ uint32_t prefix, want;
  __shared__ float cv[TOPK_MAX];
  __shared__ uint32_t ci[TOPK_MAX];
  __shared__ unsigned n_gt, n_eq_taken;
  const int tid = threadIdx.x;
  // radix select: the key of the k-th largest element
  if (tid == 0) { prefix = 0; want = k; }
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t pmask = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
    for (int i = tid; i < n_vocab; i += blockDim.x) {
      const uint32_t key = order_key(logits[i]);
      if ((key & pmask) == (prefix & pmask)) atomicAdd(&hist[(key >> shift) & 0xff], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t w = want;
      int d = 255;
      for (; d > 0; --d) {
        if (hist[d] >= w) break;
        w -= hist[d];
      }
      prefix |= (uint32_t)d << shift;
      want = w;
    }
    __syncthreads();
  }
  // candidates: keys above the threshold, then equal keys in index order
  if (tid == 0) { n_gt = 0; n_eq_taken = 0; }
  __syncthreads();
  const uint32_t T = prefix;
  for (int i = tid; i < n_vocab; i += blockDim.x) {
    const uint32_t key = order_key(logits[i]);
    if (key > T) {
      const unsigned slot = atomicAdd(&n_gt, 1u);
      cv[slot] = logits[i];
      ci[slot] = i;
    }
  }
  __syncthreads();
  if (tid == 0) {  // equal keys: lowest indices first (stable selection)
    unsigned slot = n_gt;
    for (int i = 0; i < n_vocab && slot < (unsigned)k; ++i)
      if (order_key(logits[i]) == T) { cv[slot] = logits[i]; ci[slot] = i; ++slot; }
    n_eq_taken = slot;
  }
  __syncthreads();
  const int n = (int)n_eq_taken;
  // bitonic sort, descending by value, ascending by index on ties
  int np = 1;
  while (np < n) np <<= 1;
  for (int i = n + tid; i < np; i += blockDim.x) { cv[i] = -CUDART_INF_F; ci[i] = 0xffffffffu; }
  __syncthreads();
  for (int size = 2; size <= np; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < np; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const bool ij = better(cv[j], ci[j], cv[i], ci[i]);  // j ranks before i
          if (ij == desc) {
            const float tv = cv[i]; cv[i] = cv[j]; cv[j] = tv;
            const uint32_t ti = ci[i]; ci[i] = ci[j]; ci[j] = ti;
          }
        }
      }
      __syncthreads();
    }
  if (tid == 0) {
    uint32_t pick = ci[0];
    const float mx = cv[0];
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) { cv[i] = expf_cr(__fdiv_rn(__fsub_rn(cv[i], mx), temperature)); sum = __fadd_rn(sum, cv[i]); }
    if (sum > 0.0f) {
      int nt = n;
      for (int i = 0; i < nt; ++i) cv[i] = __fdiv_rn(cv[i], sum);
      if (top_p < 1.0f) {
        float cum = 0.0f;
        for (int i = 0; i < nt; ++i) { cum = __fadd_rn(cum, cv[i]); if (cum >= top_p) { nt = i + 1; break; } }
        float s2 = 0.0f;
        for (int i = 0; i < nt; ++i) s2 = __fadd_rn(s2, cv[i]);
        if (s2 > 0.0f) for (int i = 0; i < nt; ++i) cv[i] = __fdiv_rn(cv[i], s2);
      }
      unsigned long long x = st->rng;
      x ^= x >> 12; x ^= x << 25; x ^= x >> 27;
      st->rng = x;
      const float r = (float)((double)((x * 0x2545F4914F6CDD1Dull) >> 40) / 16777216.0);
      float cum = 0.0f;
      pick = ci[nt - 1];
      for (int i = 0; i < nt; ++i) { cum = __fadd_rn(cum, cv[i]); if (r <= cum) { pick = ci[i]; break; } }
    }
    st->token = pick;
    if (token_out) *token_out = pick;
    if (ring) { ring[st->n_out % ring_cap] = pick; st->n_out++; }
  }
  __syncthreads();
  if (restore) {
    const int nh = st->hist_len;
    for (int i = tid; i < nh; i += blockDim.x) {
      const uint32_t tok = st->hist[i];
      bool first = tok < (uint32_t)n_vocab;
      for (int j = 0; j < i && first; ++j) first = st->hist[j] != tok;
      if (first) logits[tok] = st->saved[i];
    }
  }
  __syncthreads();
  if (accept && tid == 0) accept_token(st, st->token);
}

// ---------------------------------------------------------------------------
// Tensor-parallel pieces. Upstream has one process and no exchange; these are
// the steps around the exchanges of the sharded decode step, each written so
// the sharded result equals the unsharded one bit for bit.

// |x| max of a vector, one CTA (the shard's contribution to the global absmax
// of upstream's quantiser, src/gemv.c:20-40)
__global__ void __launch_bounds__(1024) amax_kernel(const float* __restrict__ v, int n, float* out) {
  __shared__ float red[32];
  float am = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) am = absmax_acc(am, v[i]);
  am = block_reduce<float>(am, red, OpMax(), 0.0f);
  if (threadIdx.x == 0) out[0] = am;
}

// Row sums of gathered block terms in upstream's block order: shard k holds
// the column blocks after those of shards 0..k-1, so rank order then block
// order is the global block order (src/gemv.c:86-95, ternary.c:236-244).
// Then the row scale (ternary: the global absmax / 127) and the residual add.
struct FoldParams {
  const float* g;      // [tp][rows][stride] gathered terms
  int tp, rows, stride, ternary;
  int count[8];        // terms per row of each shard
  const float* amax;   // ternary: global absmax
  float* x;            // residual, += the row values
};

__global__ void fold_kernel(const FoldParams f) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= f.rows) return;
  float acc = 0.0f;
  for (int k = 0; k < f.tp; ++k) {
    const float* t = f.g + ((size_t)k * f.rows + r) * f.stride;
    for (int j = 0; j < f.count[k]; ++j) acc = __fadd_rn(acc, t[j]);
  }
  float v = acc;
  if (f.ternary) {
    const float amax = *f.amax;
    v = __fmul_rn(acc, amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 0.0f);
  }
  f.x[r] = __fadd_rn(f.x[r], v);
}

// This shard's best logit (first strict maximum, ties to the lowest index,
// src/sample.c:147-153) as {value, global index bits}.
__global__ void __launch_bounds__(1024) tp_argmax_kernel(const float* __restrict__ logits, int n,
                                                         uint32_t offset, float* best) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  float bv = -CUDART_INF_F;
  uint32_t bi = 0xffffffffu;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (better(logits[i], offset + i, bv, bi)) { bv = logits[i]; bi = offset + i; }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
    best[0] = bv;
    best[1] = __uint_as_float(bi);
  }
}

// Repeat penalty on a shard's vocabulary rows [vocab0, vocab0 + n): each
// distinct history token whose row lives here is penalised as
// penalty_kernel does (src/sample.c:95-107), at its local index. Every shard
// holds the same history (every shard accepts the same picks), so the
// shards together penalise exactly the logits the unsplit sampler does.
FOX_DEV bool tp_hist_first(const SamplerDev* st, int i, uint32_t vocab0, int n) {
  const uint32_t tok = st->hist[i];
  bool first = tok >= vocab0 && tok - vocab0 < (uint32_t)n;
  for (int j = 0; j < i && first; ++j) first = st->hist[j] != tok;
  return first;
}

__global__ void tp_penalty_kernel(SamplerDev* st, float* logits, int n, uint32_t vocab0, float penalty) {
  const int h = st->hist_len;
  for (int i = threadIdx.x; i < h; i += blockDim.x) {
    if (!tp_hist_first(st, i, vocab0, n)) continue;
    const uint32_t tok = st->hist[i];
    int c = 0;
    for (int j = 0; j < h; ++j) c += st->hist[j] == tok;
    float v = logits[tok - vocab0];
    st->saved[i] = v;
    for (int r = 0; r < c; ++r) v = v > 0.0f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
    logits[tok - vocab0] = v;
  }
}

__global__ void tp_restore_kernel(SamplerDev* st, float* logits, int n, uint32_t vocab0) {
  for (int i = threadIdx.x; i < (int)st->hist_len; i += blockDim.x)
    if (tp_hist_first(st, i, vocab0, n)) logits[st->hist[i] - vocab0] = st->saved[i];
}

__global__ void tp_accept_kernel(SamplerDev* st, const uint32_t* token) {
  if (threadIdx.x == 0 && blockIdx.x == 0) accept_token(st, *token);
}

// The winner over all shards' {value, index} pairs becomes the next token.
__global__ void tp_pick_kernel(const float* __restrict__ pairs, int tp, uint32_t* token,
                               uint32_t* ring, int ring_cap, const int* pos) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float bv = -CUDART_INF_F;
  uint32_t bi = 0xffffffffu;
  for (int k = 0; k < tp; ++k) {
    const float v = pairs[2 * k];
    const uint32_t i = __float_as_uint(pairs[2 * k + 1]);
    if (better(v, i, bv, bi)) { bv = v; bi = i; }
  }
  if (bi == 0xffffffffu) bi = 0;  // all NaN: upstream keeps index 0
  token[0] = bi;
  if (ring) ring[(*pos) % ring_cap] = bi;
}

}  // namespace fox
