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

// K/V cache rows of one layer. Contiguous: [kv_head][n_ctx][hd]. Paged (a
// block table given): position p of a sequence lives in physical page
// table[p / KV_PAGE] of the layer's page pool, and a page holds KV_PAGE
// positions of every KV head, [kv_head][KV_PAGE][hd]. The row of (kvh, p),
// in units of hd elements.
constexpr int KV_PAGE = 64;
FOX_DEV size_t kv_row(const int* table, int n_ctx, int n_kv, int kvh, int pos) {
  if (!table) return (size_t)kvh * n_ctx + pos;
  return ((size_t)__ldg(table + (pos >> 6)) * n_kv + kvh) * KV_PAGE + (pos & (KV_PAGE - 1));
}

// e^x in binary32 as upstream gets it from glibc's expf (glibc >= 2.27: the
// published ARM optimized-routines algorithm; x86-64 hosts with FMA run its
// FMA build). With N = 32:
//   z = x * N/ln2; k = round(z) by adding and subtracting 1.5 * 2^52, the
//   sum formed with one fused multiply-add; r = x * N/ln2 - k, another;
//   2^(k/N) = the table entry 2^((k mod N)/N), its exponent field lowered by
//   (k mod N) * 2^52 / N, plus k * 2^52 / N in the bits;
//   e^x = 2^(k/N) * (1 + c2 r + (c1 + c0 r) r^2), in double with fused
//   multiply-adds, rounded once to float.
// c0..c2 are the algorithm's published coefficients of 2^(r/N) (those of
// 2^u scaled by N^-3, N^-2, N^-1); the table is 2^(i/N) rounded to double.
// |x| >= 88: -inf gives 0, inf and NaN x + x, x above ln(2^128) inf, x
// below ln(2^-150) 0, the rest the main path. Bit-identical to the host's
// libm expf at every float in [-104, 89] (checked exhaustively).
// In global memory, read through the read-only cache: lanes index it by
// their own k mod 32, which constant memory would serialise.
__device__ const uint64_t kExpTab[32] = {
    0x3ff0000000000000ull,
    0x3fefd9b0d3158574ull,
    0x3fefb5586cf9890full,
    0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull,
    0x3fef54873168b9aaull,
    0x3fef387a6e756238ull,
    0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull,
    0x3feef1a7373aa9cbull,
    0x3feedea64c123422ull,
    0x3feece086061892dull,
    0x3feebfdad5362a27ull,
    0x3feeb42b569d4f82ull,
    0x3feeab07dd485429ull,
    0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull,
    0x3fee9f75e8ec5f74ull,
    0x3feea11473eb0187ull,
    0x3feea589994cce13ull,
    0x3feeace5422aa0dbull,
    0x3feeb737b0cdc5e5ull,
    0x3feec49182a3f090ull,
    0x3feed503b23e255dull,
    0x3feee89f995ad3adull,
    0x3feeff76f2fb5e47ull,
    0x3fef199bdd85529cull,
    0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull,
    0x3fef7c97337b9b5full,
    0x3fefa4afa2a490daull,
    0x3fefd0765b6e4540ull};

FOX_DEV float expf_up(float x) {
  const uint32_t ux = __float_as_uint(x);
  const uint32_t abstop = (ux >> 20) & 0x7ffu;
  if (abstop >= 0x42bu) {  // |x| >= 88, or NaN
    if (ux == 0xff800000u) return 0.0f;
    if (abstop >= 0x7f8u) return __fadd_rn(x, x);
    if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);
    if (x < -0x1.9fe368p6f) return 0.0f;
  }
  constexpr double kN = 32.0;
  constexpr double kInvLn2N = 0x1.71547652b82fep+0 * kN;
  constexpr double kShift = 0x1.8p+52;
  constexpr double kC0 = 0x1.c6af84b912394p-5 / kN / kN / kN;
  constexpr double kC1 = 0x1.ebfce50fac4f3p-3 / kN / kN;
  constexpr double kC2 = 0x1.62e42ff0c52d6p-1 / kN;
  const double xd = (double)x;
  const double kz = __fma_rn(kInvLn2N, xd, kShift);
  const uint64_t ki = (uint64_t)__double_as_longlong(kz);
  const double kd = __dsub_rn(kz, kShift);
  const double r = __fma_rn(kInvLn2N, xd, -kd);
  const uint64_t t = __ldg(reinterpret_cast<const unsigned long long*>(kExpTab) + (ki % 32)) + (ki << 47);
  const double sc = __longlong_as_double((long long)t);
  const double z = __fma_rn(kC0, r, kC1);
  const double r2 = __dmul_rn(r, r);
  double y = __fma_rn(kC2, r, 1.0);
  y = __fma_rn(z, r2, y);
  return __double2float_rn(__dmul_rn(y, sc));
}

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
