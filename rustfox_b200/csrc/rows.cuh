// Row-per-lane Q8_0 GEMV for the output head (sm_100a).
//
// Upstream's head is fox_gemv on Q8_0 weights with float activations
// (src/kernels.c:98-113, 709-718): per row, per 32-element block in order,
// s = sum over the block's elements in order of q_j * x_j (a multiply and an
// add, each rounded), then acc += d * s. Every operation of that chain is
// serial within the row. The bit-exact device form gives each lane whole
// rows: no shared-memory term buffer, no block barrier inside the loop, and
// the row's float chain runs in registers in upstream's order.
//
// Each lane owns two rows, lane r of the unit pair (2u, 2u+1) of 32-row
// units, and advances both chains together (two independent dependency
// chains per thread). int8 -> float is a byte_perm into the mantissa of 2^23
// and one exact subtraction, done for both rows by one paired fp32 add
// (add.rn.f32x2) of sm_100.
//
// Layout (pack_q8_rows32_kernel): units of 32 rows; inside a unit, block b of
// row r has its qs[0..16) at plane 0 [b][r], qs[16..32) at plane 1 [b][r]
// and its fp16 scale at plane 2 [b][r], so a warp's load of one block of its
// 32 rows is one contiguous 512-byte (or 64-byte) run.
#pragma once

#include "gemv.cuh"

namespace fox {

FOX_DEV unsigned long long f2pack(float a, float b) {
  return (unsigned long long)__float_as_uint(a) | ((unsigned long long)__float_as_uint(b) << 32);
}
FOX_DEV float f2lo(unsigned long long v) { return __uint_as_float((uint32_t)v); }
FOX_DEV float f2hi(unsigned long long v) { return __uint_as_float((uint32_t)(v >> 32)); }
FOX_DEV unsigned long long fadd2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

constexpr int ROWS_THREADS = 256;

// one block of two rows: qs as 8 words each, d as fp16 bits
struct Q8Pair { uint4 a0, a1, b0, b1; uint16_t da, db; };

FOX_DEV void q8_load(Q8Pair& r, const uint8_t* ua, const uint8_t* ub, int nb, int b, int lane, bool has_b) {
  const size_t o = ((size_t)b * 32 + lane) * 16;
  r.a0 = ldg_stream16(ua + o);
  r.a1 = ldg_stream16(ua + (size_t)nb * 512 + o);
  r.da = ldg_stream2(ua + (size_t)nb * 1024 + ((size_t)b * 32 + lane) * 2);
  if (has_b) {
    r.b0 = ldg_stream16(ub + o);
    r.b1 = ldg_stream16(ub + (size_t)nb * 512 + o);
    r.db = ldg_stream2(ub + (size_t)nb * 1024 + ((size_t)b * 32 + lane) * 2);
  } else {
    r.b0 = r.b1 = make_uint4(0, 0, 0, 0);
    r.db = 0;
  }
}

// s = sum_j q_j * x_j for both rows, j in order. The paired add only turns
// the two rows' int8 codes into floats (exact: no multiply it could be fused
// with); the chain itself is scalar __fmul_rn / __fadd_rn, which the
// compiler never contracts into a fused multiply-add.
FOX_DEV void q8_block(const Q8Pair& r, const float* xs, float& sa, float& sb) {
  const uint32_t wa[8] = {r.a0.x, r.a0.y, r.a0.z, r.a0.w, r.a1.x, r.a1.y, r.a1.z, r.a1.w};
  const uint32_t wb[8] = {r.b0.x, r.b0.y, r.b0.z, r.b0.w, r.b1.x, r.b1.y, r.b1.z, r.b1.w};
  const unsigned long long magic = f2pack(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
  sa = 0.0f;
  sb = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t va = wa[w] ^ 0x80808080u, vb = wb[w] ^ 0x80808080u;
    const float4 x = reinterpret_cast<const float4*>(xs)[w];
    const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const unsigned long long q = fadd2(f2pack(__uint_as_float(__byte_perm(va, 0x4B000000u, 0x7540 + k)),
                                                __uint_as_float(__byte_perm(vb, 0x4B000000u, 0x7540 + k))),
                                         magic);
      sa = __fadd_rn(sa, __fmul_rn(f2lo(q), xv[k]));
      sb = __fadd_rn(sb, __fmul_rn(f2hi(q), xv[k]));
    }
  }
}

// DEPTH: blocks of look-ahead per warp (1, or 2 for twice the bytes in flight
// at the same occupancy; the arithmetic is the same).
template <int PRO, int DEPTH = 1>
__global__ void __launch_bounds__(ROWS_THREADS) q8_rows_kernel(const GemvParams p) {
  static_assert(DEPTH == 1 || DEPTH == 2, "look-ahead");
  griddep_launch_dependents();
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31;
  const int K = p.K, nb = p.nb;
  float* xs = reinterpret_cast<float*>(smem);  // the activations, K floats
  double* red = reinterpret_cast<double*>(smem + (size_t)K * 4);
  const int units = p.n_rows / 32;
  const int pairs = (units + 1) / 2;
  const int warps = nth >> 5;
  const size_t unit_bytes = (size_t)32 * nb * 34;
  int pu = blockIdx.x * warps + (tid >> 5);

  // the first block(s) of this warp's first rows are requested before the wait
  Q8Pair cur, nxt, nxt2;
  if (pu < pairs) {
    const bool hb = 2 * pu + 1 < units;
    const uint8_t* ua = p.w + (size_t)(2 * pu) * unit_bytes;
    q8_load(cur, ua, ua + unit_bytes, nb, 0, lane, hb);
    if (DEPTH == 2 && nb > 1) q8_load(nxt, ua, ua + unit_bytes, nb, 1, lane, hb);
  }
  griddep_wait();

  // activations: (RMSNorm'd) x
  double ss = 0.0;
  for (int i = tid; i < K; i += nth) {
    const float v = p.x[i];
    if (PRO == PRO_NORM) ss += (double)v * (double)v;
    xs[i] = v;
  }
  if (PRO == PRO_NORM) {
    const double sum = block_reduce<double>(ss, red, OpAddD(), 0.0);
    const float scale = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)K), (double)p.eps)));
    for (int i = tid; i < K; i += nth) xs[i] = __fmul_rn(__fmul_rn(xs[i], scale), p.norm_w[i]);
  }
  __syncthreads();

  for (; pu < pairs; pu += gridDim.x * warps) {
    const bool hb = 2 * pu + 1 < units;
    const uint8_t* ua = p.w + (size_t)(2 * pu) * unit_bytes;
    const uint8_t* ub = ua + unit_bytes;
    float acca = 0.0f, accb = 0.0f;
    for (int b = 0; b < nb; ++b) {
      if (DEPTH == 1) {
        if (b + 1 < nb) q8_load(nxt, ua, ub, nb, b + 1, lane, hb);
      } else {
        if (b + 2 < nb) q8_load(nxt2, ua, ub, nb, b + 2, lane, hb);
      }
      float sa, sb;
      q8_block(cur, xs + (size_t)b * 32, sa, sb);
      acca = __fadd_rn(acca, __fmul_rn(h2f(cur.da), sa));
      accb = __fadd_rn(accb, __fmul_rn(h2f(cur.db), sb));
      if (b + 1 < nb) cur = nxt;
      if (DEPTH == 2 && b + 2 < nb) nxt = nxt2;
    }
    p.out[(size_t)(2 * pu) * 32 + lane] = acca;
    if (hb) p.out[(size_t)(2 * pu + 1) * 32 + lane] = accb;
    const int pn = pu + gridDim.x * warps;
    if (pn < pairs) {
      const bool hn = 2 * pn + 1 < units;
      const uint8_t* na = p.w + (size_t)(2 * pn) * unit_bytes;
      q8_load(cur, na, na + unit_bytes, nb, 0, lane, hn);
      if (DEPTH == 2 && nb > 1) q8_load(nxt, na, na + unit_bytes, nb, 1, lane, hn);
    }
  }
}

}  // namespace fox
