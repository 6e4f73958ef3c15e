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

// QKV[t] holds the q, k and v rows of token t (position pos0 + t). Adjacent
// row pairs of q and k are rotated with the position's tables; q goes to
// Q[t], k and v to the caches ([kv_head][n_ctx][hd], f16 or f32).
__global__ void qkv_rows_kernel(const float* __restrict__ QKV, int n_rows, int nq, int nkv, int hd,
                                int n_ctx, int pos0, const float* __restrict__ rope_cos,
                                const float* __restrict__ rope_sin, int kv_f16, void* kcache,
                                void* vcache, float* __restrict__ Q) {
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
        const size_t idx = ((size_t)(rr / hd) * n_ctx + P) * hd + rr % hd;
        if (kv_f16) reinterpret_cast<__half*>(kcache)[idx] = __float2half_rn(o);
        else reinterpret_cast<float*>(kcache)[idx] = o;
      }
    } else {
      const int rr = rg - nq - nkv;
      const size_t idx = ((size_t)(rr / hd) * n_ctx + P) * hd + rr % hd;
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
    H[(size_t)t * F + k] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf_cr(-g))), up);
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

}  // namespace fox
