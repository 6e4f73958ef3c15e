// Shared device helpers for libfoxcuda (sm_100a).
//
// Float arithmetic that must round exactly like upstream RustFox's C (built
// without FMA contraction) goes through the explicit-rounding intrinsics
// (__fmul_rn / __fadd_rn / __fsub_rn / __fdiv_rn), which nvcc never fuses.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define FOX_DEV __device__ __forceinline__

namespace fox {

// ggml type ids (upstream include/fox/fox.h:203-213)
enum GgmlType : int {
  T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14, T_TQ1_0 = 34, T_TQ2_0 = 35
};

// bytes per block / elements per block (upstream src/gguf.c:160-195)
__host__ __device__ constexpr int block_bytes(int t) {
  return t == T_TQ1_0 ? 54 : t == T_TQ2_0 ? 66 : t == T_Q8_0 ? 34 : t == T_Q4_K ? 144
       : t == T_Q6_K ? 210 : t == T_F16 ? 2 : 4;
}
__host__ __device__ constexpr int block_elems(int t) {
  return (t == T_Q8_0) ? 32 : (t == T_F32 || t == T_F16) ? 1 : 256;
}

// Exact binary16 -> binary32 (upstream src/kernels.c:14-39 is exact too).
FOX_DEV float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

FOX_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
FOX_DEV double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
FOX_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide reductions through a small shared scratch (>= 32 entries).
// Every thread of the block must call them; all get the result.
template <typename T, typename Op>
FOX_DEV T block_reduce(T v, T* scratch, Op op, T init) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();  // scratch may still be read by a previous reduction
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  T r = init;
  for (int i = 0; i < nwarps; ++i) r = op(r, scratch[i]);
  return r;
}

struct OpMax { FOX_DEV float operator()(float a, float b) const { return fmaxf(a, b); } };
struct OpAddD { FOX_DEV double operator()(double a, double b) const { return a + b; } };
struct OpAddF { FOX_DEV float operator()(float a, float b) const { return a + b; } };

// One int8 activation with upstream's rounding (src/gemv.c:113-119 and
// src/kernels.c:745-751): v = x * inv, half away from zero, truncate, clamp.
FOX_DEV int quant1(float x, float inv) {
  float v = __fmul_rn(x, inv);
  float r = v < 0.0f ? __fsub_rn(v, 0.5f) : __fadd_rn(v, 0.5f);
  int q = __float2int_rz(r);
  return q > 127 ? 127 : (q < -127 ? -127 : q);
}

FOX_DEV uint32_t pack4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) |
         ((uint32_t)(d & 0xff) << 24);
}

FOX_DEV int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// Correctly rounded e^x in binary32: the double-precision exp rounded once to
// float (the double result is within an ulp of e^x, far inside the float
// rounding interval except at measure-zero ties). Upstream calls glibc's expf,
// which differs from the correctly rounded value on about 7.6e-5 of the
// inputs in [-104, 89]; the oracle can run with either (or_set_exp_mode).
FOX_DEV float expf_cr(float x) { return (float)exp((double)x); }

// |x| max that ignores NaN the way upstream's `if (a > amax)` does.
FOX_DEV float absmax_acc(float amax, float x) {
  float a = fabsf(x);
  return a > amax ? a : amax;
}

// Loads that stream weights once: keep them out of L1.
FOX_DEV uint4 ldg_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
FOX_DEV uint32_t ldg_stream4(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
FOX_DEV uint16_t ldg_stream2(const void* p) {
  uint16_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

}  // namespace fox
