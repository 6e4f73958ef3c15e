// M-token ternary GEMM on the 5th-generation tensor cores (tcgen05, kind::i8).
//
// Upstream's forward_batch runs one GEMV per token (src/forward.c:188-213):
// each token's activations are quantised with their own absmax scale
// (src/gemv.c:11-42) and every output row is
//     acc = 0.0f; for each 256-wide block b in order: acc += d_b * (float)S_b;
//     out = acc * act_scale
// where S_b is the exact int32 sum of (code - 1) * q over the block
// (src/gemv.c:155-192, src/ternary.c:253-287,303-325). For M tokens these
// block sums are one int8 contraction per block: D[row][token] = W_b . X_b^T.
//
// One CTA owns 128 weight rows (the MMA's M) and NT tokens (its N). Per block:
//   1. all threads decode the block's 2-bit codes of the 128 rows to int8
//      (code - 1) and copy the NT tokens' int8 activations into shared memory,
//      both in the no-swizzle K-major core-matrix layout (8 rows x 16 bytes);
//   2. one thread issues eight 128 x NT x 32 MMAs into a TMEM accumulator and
//      commits them to an mbarrier;
//   3. all threads read the previous block's int32 sums from TMEM
//      (tcgen05.ld, one row per thread) and fold them in float exactly as the
//      GEMV does.
// Shared-memory operands and TMEM accumulators are double-buffered, so the
// MMAs of block b run while block b-1 is folded and block b+1's bytes load.
// Integer sums are exact and the fold order is upstream's, so every token's
// output is bit-identical to the single-token GEMV.
//
// Weights come in the library's packed layout (pack.cuh): units of U rows,
// four 16-byte planes of qs per block then the fp16 scales. The block scales
// of the CTA's 128 rows are staged in shared memory once.
//
// Every wait is bounded. On a timeout the CTA records it in p.err, waits
// (bounded) for its last commit, frees its TMEM and returns.
#pragma once

#include "common.cuh"

namespace fox {

constexpr int TC_ROWS = 128;     // weight rows per CTA (the MMA's M)
constexpr int TC_THREADS = 256;  // 8 warps: warp w reads TMEM lanes 32*(w%4).., column half w/4
constexpr int TC_MAX_NB = 256;   // blocks per row (K <= 65536): bounds the staged scales

struct TcParams {
  const uint8_t* w;    // packed TQ2_0, U rows per unit
  const int8_t* xq;    // [n_tok][K] int8 activations
  const float* xs;     // [n_tok] activation scales
  float* out;          // [n_tok][n_rows]
  int n_rows, K, nb, U, n_tok;
  int* err;            // set to 1 when a wait gave up (may be null)
};

__host__ __device__ constexpr int tc_a_bytes() { return TC_ROWS * 256; }
__host__ __device__ constexpr int tc_b_bytes(int NT) { return NT * 256; }
__host__ __device__ constexpr int tc_tmem_cols(int NT) { return 2 * NT < 32 ? 32 : 2 * NT; }
inline size_t tc_smem_bytes(int NT, int nb) {
  return 2 * (size_t)tc_a_bytes() + 2 * (size_t)tc_b_bytes(NT) + (size_t)TC_ROWS * nb * 2;
}

// ---- tcgen05 / TMEM primitives (PTX ISA 8.6+, sm_100a) -------------------
FOX_DEV void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
FOX_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
FOX_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
FOX_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
FOX_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// generic-proxy shared-memory writes become visible to the tensor core
FOX_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor: no swizzle, K-major. lbo = byte distance
// of the two 16-byte K halves of one MMA, sbo = byte distance of consecutive
// 8-row groups. Bits 46-47 = 1 (the sm_100 descriptor version).
FOX_DEV uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::i8: s32 accumulator (bits 4-5 = 2), A and B
// signed (bits 7-9, 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at 24.
__host__ __device__ constexpr uint32_t tc_idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
FOX_DEV void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;  // no output lane disabled
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}
FOX_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
FOX_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// C consecutive 32-bit TMEM columns of this thread's lane (32x32b shape)
template <int C> struct TmemLd;
template <> struct TmemLd<4> {
  FOX_DEV static void run(uint32_t a, uint32_t* v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(a));
  }
};
template <> struct TmemLd<8> {
  FOX_DEV static void run(uint32_t a, uint32_t* v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                   "=r"(v[7])
                 : "r"(a));
  }
};
template <> struct TmemLd<16> {
  FOX_DEV static void run(uint32_t a, uint32_t* v) {
    TmemLd<8>::run(a, v);
    TmemLd<8>::run(a + 8, v + 8);
  }
};
template <> struct TmemLd<32> {
  FOX_DEV static void run(uint32_t a, uint32_t* v) {
    TmemLd<16>::run(a, v);
    TmemLd<16>::run(a + 16, v + 16);
  }
};

// (code | 0x80) - 1, then ^ 0x80: code - 1 in every byte, no borrow across bytes
FOX_DEV uint32_t codes_to_i8(uint32_t c) { return ((c | 0x80808080u) - 0x01010101u) ^ 0x80808080u; }

// DEPTH: K blocks whose weights and activations are in flight in registers
// (1: the next block only). Deeper queues overlap more global-load round
// trips with the MMAs and folds; the data, the MMAs and the fold are the same.
template <int NT, int DEPTH = 1>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_tq2_kernel(const TcParams p) {
  static_assert(NT == 8 || NT == 16 || NT == 32 || NT == 64, "token tile");
  static_assert(DEPTH == 1 || DEPTH == 2 || DEPTH == 4, "look-ahead");
  constexpr int HALF = NT / 2;                    // TMEM columns read per thread
  constexpr int BV = (NT * 16 + TC_THREADS - 1) / TC_THREADS;  // 16-byte activation pieces per thread
  constexpr uint32_t NCOLS = tc_tmem_cols(NT);
  constexpr uint32_t IDESC = tc_idesc_i8(TC_ROWS, NT);

  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_sh;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int R0 = blockIdx.x * TC_ROWS, T0 = blockIdx.y * NT;
  const int nb = p.nb, U = p.U, n_rows = p.n_rows;
  uint8_t* sA = smem;
  uint8_t* sB = smem + 2 * tc_a_bytes();
  uint16_t* sD = reinterpret_cast<uint16_t*>(smem + 2 * tc_a_bytes() + 2 * tc_b_bytes(NT));

  if (warp == 0) {
    tmem_alloc(&tmem_sh, NCOLS);
    tmem_relinquish();
  }
  if (tid == 32) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_fence_init();
  }
  // block scales of the tile's rows: sD[m * nb + b]
  for (int i = tid; i < TC_ROWS * nb; i += TC_THREADS) {
    const int m = i / nb, b = i - m * nb, r = R0 + m;
    uint16_t d = 0;
    if (r < n_rows) {
      const int u = r / U, ru = min(U, n_rows - u * U);
      const size_t base = (size_t)u * U * nb * 66, count = (size_t)ru * nb;
      d = __ldg(reinterpret_cast<const unsigned short*>(p.w + base + count * 64 +
                                                        ((size_t)(r - u * U) * nb + b) * 2));
    }
    sD[i] = d;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;

  // this thread's two (row, plane) pieces of the weight tile
  // (block 0's 16 bytes of that plane; block b is 16 * b further on)
  const uint8_t* wrow[2];
  int mrow[2], plane[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = tid + j * TC_THREADS;
    mrow[j] = i & (TC_ROWS - 1);
    plane[j] = i >> 7;
    const int r = R0 + mrow[j];
    wrow[j] = nullptr;
    if (r < n_rows) {
      const int u = r / U, ru = min(U, n_rows - u * U);
      const size_t base = (size_t)u * U * nb * 66, count = (size_t)ru * nb;
      wrow[j] = p.w + base + count * 16 * plane[j] + (size_t)(r - u * U) * nb * 16;
    }
  }
  // one K block's pieces of this thread: weights (two planes) and activations
  struct Blk { uint4 ra[2], rb[BV]; };
  auto load_block = [&](Blk& q, int b) {
    // rows past the matrix get code 1 (weight 0) at every level: 0b01010101
#pragma unroll
    for (int j = 0; j < 2; ++j)
      q.ra[j] = wrow[j] ? __ldg(reinterpret_cast<const uint4*>(wrow[j] + (size_t)b * 16))
                        : make_uint4(0x55555555u, 0x55555555u, 0x55555555u, 0x55555555u);
#pragma unroll
    for (int j = 0; j < BV; ++j) {
      const int i = tid + j * TC_THREADS;
      const int n = i % NT, c = i / NT;  // token fastest: conflict-free 16-byte stores
      q.rb[j] = make_uint4(0, 0, 0, 0);
      if (i < NT * 16 && T0 + n < p.n_tok)
        q.rb[j] = __ldg(reinterpret_cast<const uint4*>(p.xq + (size_t)(T0 + n) * p.K + (size_t)b * 256 + c * 16));
    }
  };
  auto store_block = [&](const Blk& q, int buf) {
    const uint4(&ra)[2] = q.ra;
    const uint4(&rb)[BV] = q.rb;
    uint8_t* a = sA + buf * tc_a_bytes();
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int m = mrow[j], pl = plane[j];
      uint8_t* dst = a + (m >> 3) * 2048 + (m & 7) * 16;
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        const int kc = (pl >> 1) * 8 + l * 2 + (pl & 1);  // 16-element K chunk of (plane, level)
        uint4 v;
        v.x = codes_to_i8((ra[j].x >> (2 * l)) & 0x03030303u);
        v.y = codes_to_i8((ra[j].y >> (2 * l)) & 0x03030303u);
        v.z = codes_to_i8((ra[j].z >> (2 * l)) & 0x03030303u);
        v.w = codes_to_i8((ra[j].w >> (2 * l)) & 0x03030303u);
        *reinterpret_cast<uint4*>(dst + kc * 128) = v;
      }
    }
    uint8_t* bsm = sB + buf * tc_b_bytes(NT);
#pragma unroll
    for (int j = 0; j < BV; ++j) {
      const int i = tid + j * TC_THREADS;
      if (i < NT * 16) {
        const int n = i % NT, c = i / NT;
        *reinterpret_cast<uint4*>(bsm + (n >> 3) * 2048 + c * 128 + (n & 7) * 16) = rb[j];
      }
    }
  };

  const int q4 = warp & 3, half = warp >> 2, m = q4 * 32 + lane;
  float acc[HALF];
#pragma unroll
  for (int j = 0; j < HALF; ++j) acc[j] = 0.0f;
  bool ok = true;
  int last = -1;  // last committed block
  auto fold = [&](int e) -> bool {
    const int eb = e & 1;
    const bool got = mbar_wait(&bars[eb], (unsigned)((e >> 1) & 1));
    if (!__syncthreads_and(got)) return false;
    tc_fence_after();
    uint32_t v[HALF];
    TmemLd<HALF>::run(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(eb * NT + half * HALF), v);
    tmem_wait_ld();
    const float d = h2f(sD[m * nb + e]);
#pragma unroll
    for (int j = 0; j < HALF; ++j) acc[j] = __fadd_rn(acc[j], __fmul_rn(d, __int2float_rn((int)v[j])));
    return true;
  };

  // queue[i] holds block b + i at the top of iteration b
  Blk queue[DEPTH];
#pragma unroll
  for (int i = 0; i < DEPTH; ++i)
    if (i < nb) load_block(queue[i], i);
  for (int b = 0; b < nb && ok; ++b) {
    const int buf = b & 1;
    store_block(queue[0], buf);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a0 = smem_u32(sA + buf * tc_a_bytes());
      const uint32_t b0 = smem_u32(sB + buf * tc_b_bytes(NT));
#pragma unroll
      for (int s = 0; s < 8; ++s)  // K = 32 bytes per MMA: chunks 2s and 2s + 1
        mma_i8(tmem + (uint32_t)(buf * NT), umma_desc(a0 + s * 256, 128, 2048),
               umma_desc(b0 + s * 256, 128, 2048), IDESC, s > 0 ? 1u : 0u);
      mma_commit(&bars[buf]);
    }
    last = b;
#pragma unroll
    for (int i = 0; i + 1 < DEPTH; ++i) queue[i] = queue[i + 1];
    if (b + DEPTH < nb) load_block(queue[DEPTH - 1], b + DEPTH);
    if (b >= 1) ok = fold(b - 1);
  }
  if (ok) ok = fold(nb - 1);

  if (ok) {
    const int r = R0 + m;
    if (r < n_rows)
#pragma unroll
      for (int j = 0; j < HALF; ++j) {
        const int t = T0 + half * HALF + j;
        if (t < p.n_tok) p.out[(size_t)t * n_rows + r] = __fmul_rn(acc[j], p.xs[t]);
      }
  } else {
    if (tid == 0 && p.err) atomicExch(p.err, 1);
    // the MMAs of the last commit (and every earlier one) may still be in flight
    if (last >= 0) mbar_wait(&bars[last & 1], (unsigned)((last >> 1) & 1));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, NCOLS);
}

// ---- split over K blocks (few tokens) ---------------------------------------
// With few tokens a matrix has few 128-row tiles, and each CTA above walks all
// K blocks of its tile one after another. The split form gives CTA z the
// blocks [z*bc, z*bc + bc) of its tile. Per block it writes each row's float
// term d_b * S_b (the same product the GEMV folds) to
// terms[b][token][row], and tc_fold_kernel then adds each row's terms in
// block order from 0.0f and scales by the token's activation scale. Every
// operation and its order is the single-token GEMV's, so the result is still
// bit-identical. The pipeline per CTA is the one of tc_tq2_kernel.
struct TcSplitParams {
  TcParams p;
  float* terms;  // [nb][n_tok][n_rows]
  int bc;        // blocks per CTA
};

template <int NT>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_tq2_split_kernel(const TcSplitParams sp) {
  static_assert(NT == 8 || NT == 16 || NT == 32 || NT == 64, "token tile");
  constexpr int HALF = NT / 2;
  constexpr int BV = (NT * 16 + TC_THREADS - 1) / TC_THREADS;
  constexpr uint32_t NCOLS = tc_tmem_cols(NT);
  constexpr uint32_t IDESC = tc_idesc_i8(TC_ROWS, NT);

  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_sh;

  const TcParams& p = sp.p;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int R0 = blockIdx.x * TC_ROWS, T0 = blockIdx.y * NT;
  const int nb = p.nb, U = p.U, n_rows = p.n_rows;
  const int b0 = blockIdx.z * sp.bc, nbc = min(sp.bc, nb - b0);  // this CTA's blocks
  uint8_t* sA = smem;
  uint8_t* sB = smem + 2 * tc_a_bytes();
  uint16_t* sD = reinterpret_cast<uint16_t*>(smem + 2 * tc_a_bytes() + 2 * tc_b_bytes(NT));

  if (warp == 0) {
    tmem_alloc(&tmem_sh, NCOLS);
    tmem_relinquish();
  }
  if (tid == 32) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_fence_init();
  }
  // block scales of the tile's rows for this CTA's blocks: sD[m * nbc + lb]
  for (int i = tid; i < TC_ROWS * nbc; i += TC_THREADS) {
    const int m = i / nbc, lb = i - m * nbc, r = R0 + m;
    uint16_t d = 0;
    if (r < n_rows) {
      const int u = r / U, ru = min(U, n_rows - u * U);
      const size_t base = (size_t)u * U * nb * 66, count = (size_t)ru * nb;
      d = __ldg(reinterpret_cast<const unsigned short*>(p.w + base + count * 64 +
                                                        ((size_t)(r - u * U) * nb + b0 + lb) * 2));
    }
    sD[i] = d;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;

  const uint8_t* wrow[2];
  int mrow[2], plane[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = tid + j * TC_THREADS;
    mrow[j] = i & (TC_ROWS - 1);
    plane[j] = i >> 7;
    const int r = R0 + mrow[j];
    wrow[j] = nullptr;
    if (r < n_rows) {
      const int u = r / U, ru = min(U, n_rows - u * U);
      const size_t base = (size_t)u * U * nb * 66, count = (size_t)ru * nb;
      wrow[j] = p.w + base + count * 16 * plane[j] + (size_t)(r - u * U) * nb * 16;
    }
  }
  uint4 ra[2], rb[BV];
  auto load_block = [&](int b) {  // b: the block's index in the row
#pragma unroll
    for (int j = 0; j < 2; ++j)
      ra[j] = wrow[j] ? __ldg(reinterpret_cast<const uint4*>(wrow[j] + (size_t)b * 16))
                      : make_uint4(0x55555555u, 0x55555555u, 0x55555555u, 0x55555555u);
#pragma unroll
    for (int j = 0; j < BV; ++j) {
      const int i = tid + j * TC_THREADS;
      const int n = i % NT, c = i / NT;
      rb[j] = make_uint4(0, 0, 0, 0);
      if (i < NT * 16 && T0 + n < p.n_tok)
        rb[j] = __ldg(reinterpret_cast<const uint4*>(p.xq + (size_t)(T0 + n) * p.K + (size_t)b * 256 + c * 16));
    }
  };
  auto store_block = [&](int buf) {
    uint8_t* a = sA + buf * tc_a_bytes();
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int m = mrow[j], pl = plane[j];
      uint8_t* dst = a + (m >> 3) * 2048 + (m & 7) * 16;
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        const int kc = (pl >> 1) * 8 + l * 2 + (pl & 1);
        uint4 v;
        v.x = codes_to_i8((ra[j].x >> (2 * l)) & 0x03030303u);
        v.y = codes_to_i8((ra[j].y >> (2 * l)) & 0x03030303u);
        v.z = codes_to_i8((ra[j].z >> (2 * l)) & 0x03030303u);
        v.w = codes_to_i8((ra[j].w >> (2 * l)) & 0x03030303u);
        *reinterpret_cast<uint4*>(dst + kc * 128) = v;
      }
    }
    uint8_t* bsm = sB + buf * tc_b_bytes(NT);
#pragma unroll
    for (int j = 0; j < BV; ++j) {
      const int i = tid + j * TC_THREADS;
      if (i < NT * 16) {
        const int n = i % NT, c = i / NT;
        *reinterpret_cast<uint4*>(bsm + (n >> 3) * 2048 + c * 128 + (n & 7) * 16) = rb[j];
      }
    }
  };

  const int q4 = warp & 3, half = warp >> 2, m = q4 * 32 + lane;
  bool ok = true;
  int last = -1;  // last committed local block
  auto emit = [&](int lb) -> bool {  // the terms of local block lb
    const int eb = lb & 1;
    const bool got = mbar_wait(&bars[eb], (unsigned)((lb >> 1) & 1));
    if (!__syncthreads_and(got)) return false;
    tc_fence_after();
    uint32_t v[HALF];
    TmemLd<HALF>::run(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(eb * NT + half * HALF), v);
    tmem_wait_ld();
    const float d = h2f(sD[m * nbc + lb]);
    const int r = R0 + m;
    if (r < n_rows)
#pragma unroll
      for (int j = 0; j < HALF; ++j) {
        const int t = T0 + half * HALF + j;
        if (t < p.n_tok)
          sp.terms[((size_t)(b0 + lb) * p.n_tok + t) * n_rows + r] = __fmul_rn(d, __int2float_rn((int)v[j]));
      }
    return true;
  };

  if (nbc > 0) load_block(b0);
  for (int lb = 0; lb < nbc && ok; ++lb) {
    const int buf = lb & 1;
    store_block(buf);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a0 = smem_u32(sA + buf * tc_a_bytes());
      const uint32_t bb0 = smem_u32(sB + buf * tc_b_bytes(NT));
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_i8(tmem + (uint32_t)(buf * NT), umma_desc(a0 + s * 256, 128, 2048),
               umma_desc(bb0 + s * 256, 128, 2048), IDESC, s > 0 ? 1u : 0u);
      mma_commit(&bars[buf]);
    }
    last = lb;
    if (lb + 1 < nbc) load_block(b0 + lb + 1);
    if (lb >= 1) ok = emit(lb - 1);
  }
  if (ok && nbc > 0) ok = emit(nbc - 1);

  if (!ok) {
    if (tid == 0 && p.err) atomicExch(p.err, 1);
    if (last >= 0) mbar_wait(&bars[last & 1], (unsigned)((last >> 1) & 1));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, NCOLS);
}

// out[t][r] = (terms[0][t][r] + terms[1][t][r] + ...) * xs[t], added in block
// order from 0.0f: the fold of the single-token GEMV.
__global__ void tc_fold_kernel(const float* __restrict__ terms, const float* __restrict__ xs, int n_rows,
                               int nb, int n_tok, float* __restrict__ out) {
  const size_t total = (size_t)n_tok * n_rows, plane = total;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    float acc = 0.0f;
    for (int b = 0; b < nb; ++b) acc = __fadd_rn(acc, terms[(size_t)b * plane + i]);
    out[i] = __fmul_rn(acc, xs[i / n_rows]);
  }
}

}  // namespace fox
