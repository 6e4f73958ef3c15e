// Prompt evaluation M tokens at a time (upstream forward_batch over a chunk,
// src/forward.c:295-409, run there as one GEMV per token per projection,
// src/forward.c:188-213). The projections go through the tensor-core pass
// (tc.cuh); the kernels here are the per-token steps between them, written
// row-wise over the chunk with exactly the arithmetic of the decode step's
// GEMV prologues and epilogues, so every token's values equal the ones the
// token-by-token decode produces:
//   quant_rows_kernel   RMSNorm (double sum of squares) or nothing, then one
//                       absmax scale per token and int8 rounding
//                       (src/ops.c:7-22, src/gemv.c:11-42);
//   qkv_rows_kernel     RoPE on q and k (src/ops.c:56-73) and the K/V cache
//                       write at the token's position (src/forward.c:346-362);
//   swiglu_rows_kernel  silu(gate) * up (src/ops.c:41-48);
//   add_rows_kernel     the residual add (src/ops.c:50-54).
// The double sum of squares is formed in a fixed thread partition, so
// quant_rows_kernel is launched with the thread count of the decode kernel
// that normalises the same vector.
#pragma once

#include "common.cuh"
#include "ops.cuh"

namespace fox {

// embedding rows of the chunk's tokens: X[t][e]
__global__ void embed_rows_kernel(int type, const uint8_t* __restrict__ table, size_t row_bytes,
                                  int n_embd, const uint32_t* __restrict__ tokens,
                                  float* __restrict__ X) {
  const int t = blockIdx.y;
  const uint8_t* row = table + (size_t)tokens[t] * row_bytes;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n_embd; e += gridDim.x * blockDim.x)
    X[(size_t)t * n_embd + e] = dequant_elem(type, row, e);
}

// One token per CTA: XQ[t] = int8 of (NORM ? rmsnorm(X[t]) * w : X[t]) and
// XS[t] its scale. Dynamic shared memory: K floats.
template <bool NORM>
__global__ void quant_rows_kernel(const float* __restrict__ X, int K, const float* __restrict__ norm_w,
                                  float eps, int8_t* __restrict__ XQ, float* __restrict__ XS) {
  extern __shared__ __align__(16) float xs[];
  __shared__ double red[32];
  const int t = blockIdx.x, tid = threadIdx.x, nth = blockDim.x;
  const float* x = X + (size_t)t * K;
  float am = 0.0f;
  double ss = 0.0;
  for (int i = tid * 4; i < K; i += nth * 4) {
    const float4 v = *reinterpret_cast<const float4*>(x + i);
    if (NORM)
      ss = ss + (double)v.x * (double)v.x + (double)v.y * (double)v.y + (double)v.z * (double)v.z +
           (double)v.w * (double)v.w;
    else
      am = absmax_acc(absmax_acc(absmax_acc(absmax_acc(am, v.x), v.y), v.z), v.w);
    *reinterpret_cast<float4*>(xs + i) = v;
  }
  if (NORM) {
    const double sum = block_reduce<double>(ss, red, OpAddD(), 0.0);
    const float scale = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)K), (double)eps)));
    for (int i = tid * 4; i < K; i += nth * 4) {
      float4 v = *reinterpret_cast<float4*>(xs + i);
      const float4 w = *reinterpret_cast<const float4*>(norm_w + i);
      v.x = __fmul_rn(__fmul_rn(v.x, scale), w.x);
      v.y = __fmul_rn(__fmul_rn(v.y, scale), w.y);
      v.z = __fmul_rn(__fmul_rn(v.z, scale), w.z);
      v.w = __fmul_rn(__fmul_rn(v.w, scale), w.w);
      *reinterpret_cast<float4*>(xs + i) = v;
      am = absmax_acc(absmax_acc(absmax_acc(absmax_acc(am, v.x), v.y), v.z), v.w);
    }
  }
  const float amax = block_reduce<float>(am, reinterpret_cast<float*>(red), OpMax(), 0.0f);
  const bool nz = amax > 0.0f;
  const float inv = nz ? __fdiv_rn(127.0f, amax) : 0.0f;
  if (tid == 0) XS[t] = nz ? __fdiv_rn(amax, 127.0f) : 0.0f;
  int8_t* q = XQ + (size_t)t * K;
  for (int i = tid * 4; i < K; i += nth * 4) {  // this thread's own elements of xs
    const float4 v = *reinterpret_cast<const float4*>(xs + i);
    *reinterpret_cast<uint32_t*>(q + i) = pack4(quant1(v.x, inv), quant1(v.y, inv), quant1(v.z, inv),
                                                quant1(v.w, inv));
  }
}

// The K-quant form (upstream quantize_activations_k, src/kernels.c:722-754):
// the same RMSNorm, then one absmax scale per 256 block, a warp per block.
// XS[t * (K / 256) + b] is block b's scale. Dynamic shared memory: K floats.
template <bool NORM>
__global__ void quant_rows_k_kernel(const float* __restrict__ X, int K, const float* __restrict__ norm_w,
                                    float eps, int8_t* __restrict__ XQ, float* __restrict__ XS) {
  extern __shared__ __align__(16) float xs[];
  __shared__ double red[32];
  const int t = blockIdx.x, tid = threadIdx.x, nth = blockDim.x;
  const float* x = X + (size_t)t * K;
  double ss = 0.0;
  for (int i = tid * 4; i < K; i += nth * 4) {
    const float4 v = *reinterpret_cast<const float4*>(x + i);
    if (NORM)
      ss = ss + (double)v.x * (double)v.x + (double)v.y * (double)v.y + (double)v.z * (double)v.z +
           (double)v.w * (double)v.w;
    *reinterpret_cast<float4*>(xs + i) = v;
  }
  if (NORM) {
    const double sum = block_reduce<double>(ss, red, OpAddD(), 0.0);
    const float scale = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)K), (double)eps)));
    for (int i = tid * 4; i < K; i += nth * 4) {
      float4 v = *reinterpret_cast<float4*>(xs + i);
      const float4 w = *reinterpret_cast<const float4*>(norm_w + i);
      v.x = __fmul_rn(__fmul_rn(v.x, scale), w.x);
      v.y = __fmul_rn(__fmul_rn(v.y, scale), w.y);
      v.z = __fmul_rn(__fmul_rn(v.z, scale), w.z);
      v.w = __fmul_rn(__fmul_rn(v.w, scale), w.w);
      *reinterpret_cast<float4*>(xs + i) = v;
    }
  }
  __syncthreads();  // a block's warp reads other threads' elements
  const int lane = tid & 31, warp = tid >> 5, nw = nth >> 5, nb = K >> 8;
  for (int b = warp; b < nb; b += nw) {
    float v[8], am = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) { v[k] = xs[b * 256 + lane * 8 + k]; am = absmax_acc(am, v[k]); }
    am = warp_max(am);
    const bool nz = am > 0.0f;
    const float inv = nz ? __fdiv_rn(127.0f, am) : 0.0f;
    uint32_t* dst = reinterpret_cast<uint32_t*>(XQ + (size_t)t * K + b * 256 + lane * 8);
    dst[0] = pack4(quant1(v[0], inv), quant1(v[1], inv), quant1(v[2], inv), quant1(v[3], inv));
    dst[1] = pack4(quant1(v[4], inv), quant1(v[5], inv), quant1(v[6], inv), quant1(v[7], inv));
    if (lane == 0) XS[(size_t)t * nb + b] = nz ? __fdiv_rn(am, 127.0f) : 0.0f;
  }
}

// QKV[t] holds the q, k and v rows of token t (position pos0 + t). Adjacent
// row pairs of q and k are rotated with the position's tables; q goes to
// Q[t], k and v to the caches (common.cuh kv_row: contiguous, or paged
// through `table`; f16 or f32).
__global__ void qkv_rows_kernel(const float* __restrict__ QKV, int n_rows, int nq, int nkv, int hd,
                                int n_ctx, int pos0, const float* __restrict__ rope_cos,
                                const float* __restrict__ rope_sin, int kv_f16, void* kcache,
                                void* vcache, const int* __restrict__ table, float* __restrict__ Q) {
  const int t = blockIdx.y, P = pos0 + t;
  const float* vals = QKV + (size_t)t * n_rows;
  for (int rg = blockIdx.x * blockDim.x + threadIdx.x; rg < n_rows; rg += gridDim.x * blockDim.x) {
    const float mine = vals[rg];
    if (rg < nq + nkv) {
      const float other = vals[rg ^ 1];
      const int rr = rg < nq ? rg : rg - nq;
      const int i = (rr % hd) >> 1;
      const float c = rope_cos[(size_t)P * (hd >> 1) + i];
      const float s = rope_sin[(size_t)P * (hd >> 1) + i];
      const bool odd = rg & 1;
      const float x0 = odd ? other : mine, x1 = odd ? mine : other;
      const float o = odd ? __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c))
                          : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      if (rg < nq) {
        Q[(size_t)t * nq + rg] = o;
      } else {
        const size_t idx = kv_row(table, n_ctx, nkv / hd, rr / hd, P) * hd + rr % hd;
        if (kv_f16) reinterpret_cast<__half*>(kcache)[idx] = __float2half_rn(o);
        else reinterpret_cast<float*>(kcache)[idx] = o;
      }
    } else {
      const int rr = rg - nq - nkv;
      const size_t idx = kv_row(table, n_ctx, nkv / hd, rr / hd, P) * hd + rr % hd;
      if (kv_f16) reinterpret_cast<__half*>(vcache)[idx] = __float2half_rn(mine);
      else reinterpret_cast<float*>(vcache)[idx] = mine;
    }
  }
}

// GU[t] holds the gate|up rows in the packed order (per unit of U rows, U/2
// gate rows then the same U/2 up rows); H[t][k] = silu(gate_k) * up_k.
__global__ void swiglu_rows_kernel(const float* __restrict__ GU, int n_rows, int U, float* __restrict__ H) {
  const int t = blockIdx.y, F = n_rows >> 1, hu = U >> 1;
  const float* gu = GU + (size_t)t * n_rows;
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < F; k += gridDim.x * blockDim.x) {
    const int u = k / hu, i = k - u * hu;
    const float g = gu[u * U + i], up = gu[u * U + hu + i];
    H[(size_t)t * F + k] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf_up(-g))), up);
  }
}

__global__ void add_rows_kernel(float* __restrict__ X, const float* __restrict__ T, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    X[i] = __fadd_rn(X[i], T[i]);
}

__global__ void positions_kernel(int* __restrict__ pos, int pos0, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) pos[i] = pos0 + i;
}

// ---- decode batches: row t is the next token of sequence t ---------------

// qkv_rows_kernel for a batch of sequences: row t's position is *pos[t] and
// its caches start at kbase[t] / vbase[t] plus layer_off bytes (paged
// through tables[t] when tables is given).
__global__ void qkv_seqs_kernel(const float* __restrict__ QKV, int n_rows, int nq, int nkv, int hd,
                                int n_ctx, int* const* __restrict__ pos, void* const* __restrict__ kbase,
                                void* const* __restrict__ vbase, size_t layer_off,
                                const int* const* __restrict__ tables,
                                const float* __restrict__ rope_cos, const float* __restrict__ rope_sin,
                                int kv_f16, float* __restrict__ Q) {
  const int t = blockIdx.y, P = *pos[t];
  const int* tab = tables ? tables[t] : nullptr;
  void* kcache = reinterpret_cast<uint8_t*>(kbase[t]) + layer_off;
  void* vcache = reinterpret_cast<uint8_t*>(vbase[t]) + layer_off;
  const float* vals = QKV + (size_t)t * n_rows;
  for (int rg = blockIdx.x * blockDim.x + threadIdx.x; rg < n_rows; rg += gridDim.x * blockDim.x) {
    const float mine = vals[rg];
    if (rg < nq + nkv) {
      const float other = vals[rg ^ 1];
      const int rr = rg < nq ? rg : rg - nq;
      const int i = (rr % hd) >> 1;
      const float c = rope_cos[(size_t)P * (hd >> 1) + i];
      const float s = rope_sin[(size_t)P * (hd >> 1) + i];
      const bool odd = rg & 1;
      const float x0 = odd ? other : mine, x1 = odd ? mine : other;
      const float o = odd ? __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c))
                          : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      if (rg < nq) {
        Q[(size_t)t * nq + rg] = o;
      } else {
        const size_t idx = kv_row(tab, n_ctx, nkv / hd, rr / hd, P) * hd + rr % hd;
        if (kv_f16) reinterpret_cast<__half*>(kcache)[idx] = __float2half_rn(o);
        else reinterpret_cast<float*>(kcache)[idx] = o;
      }
    } else {
      const int rr = rg - nq - nkv;
      const size_t idx = kv_row(tab, n_ctx, nkv / hd, rr / hd, P) * hd + rr % hd;
      if (kv_f16) reinterpret_cast<__half*>(vcache)[idx] = __float2half_rn(mine);
      else reinterpret_cast<float*>(vcache)[idx] = mine;
    }
  }
}

__global__ void gather_tokens_kernel(uint32_t* const* __restrict__ src, int n, uint32_t* __restrict__ dst) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = *src[i];
}

__global__ void advance_all_kernel(int* const* __restrict__ pos, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) *pos[i] += 1;
}

// splitmix64 (Steele, Lea and Flood, 2014): a counter-based 64-bit mix
FOX_DEV uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Seeded normal values (Box-Muller on the two halves of splitmix64 of the
// logical element index, layer-major [layer][kv_head][n_ctx][hd]) for
// positions [0, n_pos) of every (layer, KV head) run of a cache, stored
// where kv_row puts them (layer_elems apart). A benchmark stand-in for a
// long prompt: upstream has no way to set its cache, so these contexts are
// not compared with it.
__global__ void fill_kv_kernel(void* cache, int kv_f16, size_t runs, int n_ctx, int hd, int n_pos,
                               int n_kv, size_t layer_elems, const int* __restrict__ table, uint64_t seed) {
  const size_t per = (size_t)n_pos * hd, total = runs * per;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t run = i / per, r = i - run * per;
    const size_t logical = run * (size_t)n_ctx * hd + r;
    const int layer = (int)(run / n_kv), kvh = (int)(run % n_kv);
    const int pos = (int)(r / hd), d = (int)(r - (size_t)pos * hd);
    const size_t idx = (size_t)layer * layer_elems + kv_row(table, n_ctx, n_kv, kvh, pos) * hd + d;
    const uint64_t h = splitmix64(seed ^ splitmix64(logical));
    const float u1 = ((float)(uint32_t)(h >> 40) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
    const float u2 = (float)(uint32_t)(h & 0xFFFFFFu) * (1.0f / 16777216.0f);   // [0, 1)
    const float v = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    if (kv_f16) reinterpret_cast<__half*>(cache)[idx] = __float2half_rn(v);
    else reinterpret_cast<float*>(cache)[idx] = v;
  }
}

}  // namespace fox
