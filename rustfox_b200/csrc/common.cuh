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

// unsigned bytes of a times signed bytes of b, accumulated
FOX_DEV int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Weight loads from global memory (read-only, streamed past L1) or, with
// SH, plain loads from a shared-memory copy of the same bytes.
template <bool SH> FOX_DEV uint4 ld16(const void* p) {
  if (SH) return *reinterpret_cast<const uint4*>(p);
  return ldg_stream16(p);
}
template <bool SH> FOX_DEV uint32_t ld4(const void* p) {
  if (SH) return *reinterpret_cast<const uint32_t*>(p);
  return ldg_stream4(p);
}
template <bool SH> FOX_DEV uint16_t ld2(const void* p) {
  if (SH) return *reinterpret_cast<const uint16_t*>(p);
  return ldg_stream2(p);
}

// mbarrier and bulk-copy helpers (PTX). A CTA copies weights from global into
// its shared memory with cp.async.bulk; completion is counted in bytes on an
// mbarrier, which the threads poll with a bounded wait.
FOX_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

FOX_DEV void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
FOX_DEV void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
FOX_DEV void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// global -> this CTA's shared memory; 16-byte aligned ends, size % 16 == 0
FOX_DEV void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
FOX_DEV bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded: gives up after about a second and reports false.
FOX_DEV bool mbar_wait(uint64_t* bar, unsigned parity) {
  for (int i = 0; i < (1 << 22); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i >= 8) __nanosleep(256);
  }
  return false;
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialisation may start before its predecessor ends; griddep_wait blocks
// until the predecessor has completed and its writes are visible, and
// griddep_launch_dependents lets the successor start early. Both are no-ops
// for kernels launched without the attribute.
FOX_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FOX_DEV void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace fox
