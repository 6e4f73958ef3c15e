// Tensor-parallel exchanges over peer memory (NVLink), in place of the four
// NCCL collectives per layer of the sharded decode step.
//
// Every rank owns an exchange arena in its own device memory, shared with the
// other ranks through CUDA IPC (plain peer loads and stores only):
//   u64 amax[2][8]    at AR_AMAX   {epoch, absmax bits} of each rank, o / down
//   u64 pick[8][2]    at AR_PICK   {epoch, value bits}, {epoch, index} of each rank
//   u32 ready[2][8]   at AR_READY  epoch at which each rank's terms are complete
//   float terms_o     at AR_TERMS  this rank's o terms   [n_embd][stride_o]
//   float terms_d     after it     this rank's down terms [n_embd][stride_d]
//   u64 sums[2][world][n_embd]     every rank's row sums of the o / down
//                                  projection, {epoch, value bits} words
// A rank writes its slot in every rank's arena (its own included) and reads
// the slots of its own arena; the block terms stay where they were written
// and are read from the owner's arena, the row sums are pushed to every
// rank and read locally.
//
// Two exchanges of a row-parallel projection:
//   terms   every rank folds all ranks' block terms in upstream's block
//           order: the sharded decode equals the single-GPU one bit for bit
//   sums    every rank pushes its rows (its blocks folded in order, times the
//           activation scale; rank 0 adds the residual) and every rank adds
//           the ranks' rows in rank order: n_embd floats per rank instead of
//           n_embd x blocks, the same value on every rank, and within
//           float rounding of the single-GPU decode (one rank: bit for bit)
// Both quantise with the absmax of the whole vector, traded in the GEMV's
// prologue, so the int8 activations are the single-GPU ones.
//
// Epochs come from the device position, ((pos + 1) << 8) | phase with phase
// 2 * layer + which + 1 (the pick is 255), so a captured step needs no host
// input and every exchange of a run has its own epoch. A rank overwrites a
// slot of the same phase only after an exchange that every rank reaches only
// after reading that slot, so no value is lost. The absmax and pick slots and
// the row sums are {epoch, value} words, each written and read in one 64-bit
// access (relaxed, system scope): a reader that sees its epoch has its value,
// with no fence on either side. The block terms of the terms exchange are
// plain floats, published behind a readiness flag (st.release.sys, read with
// ld.acquire.sys). Every wait gives up after about a second, sets the
// context's error word and lets the kernel finish.
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace fox {

constexpr int TPX_MAX = 8;
constexpr size_t AR_AMAX = 0, AR_PICK = 128, AR_READY = 256, AR_TERMS = 1024;

struct XParams {
  uint8_t* peers[TPX_MAX];  // every rank's arena, mapped here (this rank's own at [rank])
  int rank, world;
  const int* pos;           // device position: the epochs
  int* err;                 // set to 2 when a wait gives up
};

FOX_DEV void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
FOX_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
FOX_DEV uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
FOX_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Self-validating words ({epoch, value} in one aligned 64-bit word, written
// and read in one access) need no fence: a reader that sees its epoch sees
// its value. Relaxed system-scope accesses keep them out of the L1 and
// let the stores leave without waiting for earlier writes.
FOX_DEV void st_relaxed_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
FOX_DEV uint64_t ld_relaxed_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
FOX_DEV void ld_volatile_v2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

FOX_DEV uint32_t tp_epoch(const int* pos, int phase) {
  return ((uint32_t)(*pos + 1) << 8) | (uint32_t)phase;
}

// An earlier wait of this context already gave up (its error word is set):
// the step is lost, so later waits give up at once instead of each running
// out its own limit.
FOX_DEV bool step_failed(const int* err) {
  return err && *reinterpret_cast<const volatile int*>(err) != 0;
}

// Bounded wait until the 32-bit word at p reaches ep (about a second), or
// until the context's error word shows the step already failed.
FOX_DEV bool wait_u32(const uint32_t* p, uint32_t ep, const int* err) {
  for (int i = 0; i < (1 << 22); ++i) {
    if (ld_acquire_sys(p) == ep) return true;
    if (i >= 16) __nanosleep(256);
    if ((i & 255) == 255 && step_failed(err)) return false;
  }
  return false;
}
FOX_DEV bool wait_hi(const uint64_t* p, uint32_t ep, uint64_t* out, const int* err) {
  for (int i = 0; i < (1 << 22); ++i) {
    const uint64_t w = ld_relaxed_sys(p);
    if ((uint32_t)(w >> 32) == ep) { *out = w; return true; }
    if (i >= 16) __nanosleep(256);
    if ((i & 255) == 255 && step_failed(err)) return false;
  }
  return false;
}

// fold_kernel (ops.cuh) reading every rank's terms from its arena once all
// ranks have signalled them: the same sums in the same order.
struct FoldXParams {
  size_t terms_off;     // byte offset of this projection's terms in an arena
  int rows, stride, ternary, which, phase;
  int count[TPX_MAX];   // terms per row of each rank
  const float* amax;    // ternary: the global absmax
  float* x;             // residual, += the row values
};

// It releases a programmatic successor at once, so that successor can stage
// its weights while this kernel waits for the peers; the successor's
// griddepcontrol.wait still waits for this whole grid and its writes.
__global__ void fold_x_kernel(const XParams x, const FoldXParams f) {
  griddep_launch_dependents();
  __shared__ int ok_sh;
  const uint32_t ep = tp_epoch(x.pos, f.phase);
  const uint32_t* ready = reinterpret_cast<const uint32_t*>(x.peers[x.rank] + AR_READY) + f.which * TPX_MAX;
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int k = 0; k < x.world && ok; ++k) ok = wait_u32(ready + k, ep, x.err);
    ok_sh = ok;
    if (!ok && x.err) atomicExch(x.err, 2);
  }
  __syncthreads();
  if (!ok_sh) return;
  // each thread's own acquire of the flags orders its reads of the terms
  for (int k = 0; k < x.world; ++k) (void)ld_acquire_sys(ready + k);
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= f.rows) return;
  float acc = 0.0f;
  for (int k = 0; k < x.world; ++k) {
    const float* t = reinterpret_cast<const float*>(x.peers[k] + f.terms_off) + (size_t)r * f.stride;
    for (int j = 0; j < f.count[k]; ++j) acc = __fadd_rn(acc, __ldcg(t + j));
  }
  float v = acc;
  if (f.ternary) {
    const float amax = *f.amax;
    v = __fmul_rn(acc, amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 0.0f);
  }
  f.x[r] = __fadd_rn(f.x[r], v);
}

// The residual completed from the sums exchange (the ranks' rows added in
// rank order, each {epoch, value} word read until it carries this
// exchange's epoch), as a kernel of its own: before the head, or where the
// next GEMV does not complete it in its prologue (gemv.cuh PRO_NFOLD, the
// same additions in the same order). Releases its successor at once.
__global__ void fold_sum_x_kernel(const XParams x, size_t y_off, int which, int phase, int n,
                                  float* __restrict__ out) {
  griddep_launch_dependents();
  const uint32_t ep = tp_epoch(x.pos, phase);
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const uint64_t* y = reinterpret_cast<const uint64_t*>(x.peers[x.rank] + y_off);
  float a = 0.0f;
  for (int k = 0; k < x.world; ++k) {
    uint64_t w = 0;
    if (!wait_hi(y + (size_t)k * n + r, ep, &w, x.err)) {
      if (x.err) atomicExch(x.err, 2);
      return;
    }
    const float v = __uint_as_float((uint32_t)w);
    a = k == 0 ? v : __fadd_rn(a, v);
  }
  out[r] = a;
}

// This rank's {value, index} (tp_argmax_kernel) published; every rank's pair
// into pairs[2k], pairs[2k + 1] for tp_pick_kernel.
__global__ void pick_x_kernel(const XParams x, const float* __restrict__ best, float* __restrict__ pairs) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint32_t ep = tp_epoch(x.pos, 255);
  const uint64_t w0 = ((uint64_t)ep << 32) | __float_as_uint(best[0]);
  const uint64_t w1 = ((uint64_t)ep << 32) | __float_as_uint(best[1]);
  for (int k = 0; k < x.world; ++k) {
    uint64_t* slot = reinterpret_cast<uint64_t*>(x.peers[k] + AR_PICK) + 2 * x.rank;
    st_relaxed_sys(slot, w0);
    st_relaxed_sys(slot + 1, w1);
  }
  const uint64_t* mine = reinterpret_cast<const uint64_t*>(x.peers[x.rank] + AR_PICK);
  for (int k = 0; k < x.world; ++k) {
    uint64_t a = 0, b = 0;
    if (!wait_hi(mine + 2 * k, ep, &a, x.err) || !wait_hi(mine + 2 * k + 1, ep, &b, x.err)) {
      if (x.err) atomicExch(x.err, 2);
      pairs[2 * k] = -CUDART_INF_F;
      pairs[2 * k + 1] = __uint_as_float(0xffffffffu);
      continue;
    }
    pairs[2 * k] = __uint_as_float((uint32_t)a);
    pairs[2 * k + 1] = __uint_as_float((uint32_t)b);
  }
}

}  // namespace fox
