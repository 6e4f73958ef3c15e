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
// a_j v_j. Two forms: attention_exact_kernel below (upstream's serial order,
// the parity mode) and the tile attention of attn.cuh (attention_tile_kernel),
// whose order the oracle restates.

struct AttnParams {
  const float* q;         // [n_head * hd], roped
  const void* kcache;     // this layer's caches (common.cuh kv_row)
  const void* vcache;
  const int* kv_table;    // block table of a paged cache (nullptr: contiguous)
  int kv_f16, n_ctx, hd, n_head, n_kv;
  int nt;                 // tile target of the tile attention (attn.cuh)
  int stage_rows;         // K/V rows per ring slot of the tile attention (set by its launch)
  int stage_slots;        // ring slots of the tile attention (set by its launch)
  const int* pos;
  float* out;             // [n_head * hd]
  float scale;
  // several sequences in one launch (grid z): sequence z reads q + z *
  // seq_stride, writes out + z * seq_stride, its position at *pos_list[z]
  // and its layer's caches at k_list[z] / v_list[z] + layer_off
  int seq_stride;
  int* const* pos_list;
  void* const* k_list;
  void* const* v_list;
  const int* const* table_list;  // per sequence, when the caches are paged
  size_t layer_off;
};

constexpr int ATTN_MAX_GQA = 8;
constexpr int ATTN_MAX_DPL = 8;  // head_dim <= 256

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
  for (int j = threadIdx.x; j < P; j += blockDim.x) {
    float s = 0.0f;
    const size_t base = kv_row(p.kv_table, p.n_ctx, p.n_kv, kvh, j) * hd;
    for (int d = 0; d < hd; ++d) {
      const size_t at = base + d;
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
  for (int j = threadIdx.x; j < P; j += blockDim.x) att[j] = expf_up(__fsub_rn(att[j], mx));
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
      const size_t at = kv_row(p.kv_table, p.n_ctx, p.n_kv, kvh, j) * hd + d;
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
  constexpr int NWARP = TOPK_THREADS / 32;
  __shared__ unsigned hist[256];
  __shared__ uint32_t prefix, want;
  __shared__ float cv[2 * TOPK_MAX];  // [0, TOPK_MAX): candidates; above: keys equal to the threshold
  __shared__ uint32_t ci[2 * TOPK_MAX];
  __shared__ unsigned n_gt, n_eq, n_eq_taken, wcount[NWARP];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // radix select: the key of the k-th largest element. The histogram adds
  // are aggregated per warp over lanes with the same digit (logits crowd a
  // few top-byte digits).
  if (tid == 0) { prefix = 0; want = k; }
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t pmask = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
    const uint32_t pre = prefix & pmask;
    for (int base = 0; base < n_vocab; base += TOPK_THREADS) {
      const int i = base + tid;
      uint32_t digit = 0xffffffffu;  // no digit: out of range or another prefix
      if (i < n_vocab) {
        const uint32_t key = order_key(logits[i]);
        if ((key & pmask) == pre) digit = (key >> shift) & 0xffu;
      }
      const unsigned peers = __match_any_sync(0xffffffffu, digit);
      if (digit != 0xffffffffu && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], (unsigned)__popc(peers));
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
  // candidates: every key above the threshold T (fewer than k), then keys
  // equal to T in index order until there are k
  if (tid == 0) { n_gt = 0; n_eq = 0; }
  __syncthreads();
  const uint32_t T = prefix;
  for (int i = tid; i < n_vocab; i += blockDim.x) {
    const float v = logits[i];
    const uint32_t key = order_key(v);
    if (key > T) {
      const unsigned slot = atomicAdd(&n_gt, 1u);
      cv[slot] = v;
      ci[slot] = i;
    } else if (key == T) {
      const unsigned slot = atomicAdd(&n_eq, 1u);
      if (slot < TOPK_MAX) { cv[TOPK_MAX + slot] = v; ci[TOPK_MAX + slot] = i; }
    }
  }
  __syncthreads();
  const unsigned need = (unsigned)k - n_gt;
  if (n_eq <= need) {
    // all of them (their order is the sort's business)
    for (unsigned j = tid; j < n_eq; j += blockDim.x) { cv[n_gt + j] = cv[TOPK_MAX + j]; ci[n_gt + j] = ci[TOPK_MAX + j]; }
    if (tid == 0) n_eq_taken = n_gt + n_eq;
  } else {
    // more equal keys than places: the lowest indices, by an ordered scan of
    // the vocabulary TOPK_THREADS ids at a time
    unsigned taken = 0;
    for (int base = 0; base < n_vocab && taken < need; base += TOPK_THREADS) {
      const int i = base + tid;
      const bool eq = i < n_vocab && order_key(logits[i]) == T;
      const unsigned bal = __ballot_sync(0xffffffffu, eq);
      if (lane == 0) wcount[warp] = (unsigned)__popc(bal);
      __syncthreads();
      unsigned off = taken, all = 0;
      for (int w = 0; w < NWARP; ++w) {
        if (w < warp) off += wcount[w];
        all += wcount[w];
      }
      off += (unsigned)__popc(bal & ((1u << lane) - 1u));
      if (eq && off < need) { cv[n_gt + off] = logits[i]; ci[n_gt + off] = i; }
      taken += all;  // the same in every thread
      __syncthreads();  // wcount is rewritten by the next block
    }
    if (tid == 0) n_eq_taken = n_gt + min(taken, need);
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
    for (int i = 0; i < n; ++i) { cv[i] = expf_up(__fdiv_rn(__fsub_rn(cv[i], mx), temperature)); sum = __fadd_rn(sum, cv[i]); }
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
