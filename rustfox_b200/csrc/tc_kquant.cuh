// M-token K-quant GEMM on the tensor cores (tcgen05 kind::i8): Q4_K and Q6_K.
//
// Upstream runs one K-quant GEMV per token (src/forward.c:188-213): the
// activations are quantised with one absmax scale per 256 block
// (src/kernels.c:722-754), and every output row is the in-order float sum of
// per-block terms:
//   Q4_K (src/kernels.c:465-500): for sub-block j (32 elements),
//       as * ((d * sc_j) * dot_j - (dmin * m_j) * sum_j)
//     with dot_j = sum nibble * q and sum_j = sum q;
//   Q6_K (src/kernels.c:531-569,636-661): for group (half, sub),
//       (as * d) * G,  G = sum_k scale[half*8 + sub + 2k] * (dot_k - 32 * s_k)
//     over four 16-element runs k, dot_k = sum q6 * q (q6 unsigned), s_k = sum q.
// The integer dots come from the tensor cores; everything else is the GEMV's
// arithmetic in the GEMV's order, so each token's row is bit-identical to
// the single-token GEMV (gemv.cuh, W<Q4_K> / W<Q6_K>).
//
// CTA: 128 weight rows (the MMA's M) x NT tokens (its N), all K blocks in
// order, operands and accumulators double-buffered as in tc.cuh.
//   Q4_K: the 4-bit codes become int8 0..15 in shared memory; eight
//         128 x NT x 32 MMAs per block, one per sub-block, each into its own
//         TMEM accumulator.
//   Q6_K: the 6-bit codes become int8 0..63. A 32-wide MMA spans two runs
//         whose scales differ, so the activations are staged twice: B0 holds
//         the first run of every 32 (the second zeroed), B1 the second.
//         Sixteen MMAs per block give the sixteen run dots.
// The per-run activation sums come from the staged int8 activations.
#pragma once

#include "tc.cuh"

namespace fox {

struct TcKParams {
  const uint8_t* w;    // packed Q4_K or Q6_K, U rows per unit
  const int8_t* xq;    // [n_tok][K] int8 activations (per-256 scales)
  const float* xs;     // [n_tok][nb] activation scales
  float* out;          // out[t * out_stride + r]
  int out_stride;
  int n_rows, K, nb, U, n_tok;
  int* err;
};

template <int T> struct KqTraits;
template <> struct KqTraits<T_Q4_K> {
  static constexpr int BB = 144;     // block bytes
  static constexpr int NACC = 8;     // accumulators per block
  static constexpr int NBV = 1;      // activation tiles
  static constexpr int RS = 16;      // per-row scale bytes staged (scales[12] as 3 words, d|dmin)
};
template <> struct KqTraits<T_Q6_K> {
  static constexpr int BB = 210;
  static constexpr int NACC = 16;
  static constexpr int NBV = 2;
  static constexpr int RS = 20;      // scales[16], d (2 bytes), pad
};

template <int T>
__host__ __device__ constexpr int tck_tmem_cols(int NT) {
  return 2 * KqTraits<T>::NACC * NT;
}
// shared memory of one buffer: A, activation tile(s), row scales, chunk sums, token scales
template <int T>
__host__ __device__ constexpr int tck_buf_bytes(int NT) {
  return tc_a_bytes() + KqTraits<T>::NBV * tc_b_bytes(NT) + TC_ROWS * KqTraits<T>::RS + NT * 16 * 4 + NT * 4;
}

// DEPTH: K blocks in flight per thread in registers, as in tc_tq2_kernel.
template <int T, int NT, int DEPTH = 1>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_kq_kernel(const TcKParams p) {
  using K = KqTraits<T>;
  static_assert(NT == 8 || NT == 16, "token tile");
  static_assert(DEPTH == 1 || DEPTH == 2 || DEPTH == 4, "look-ahead");
  constexpr int HALF = NT / 2;
  constexpr int BV = (NT * 16 + TC_THREADS - 1) / TC_THREADS;
  constexpr uint32_t NCOLS = tck_tmem_cols<T>(NT);
  static_assert(NCOLS == 128 || NCOLS == 256, "TMEM allocation");
  constexpr uint32_t IDESC = tc_idesc_i8(TC_ROWS, NT);
  constexpr int BUF = tck_buf_bytes<T>(NT);
  constexpr int OFF_B = tc_a_bytes();
  constexpr int OFF_RS = OFF_B + K::NBV * tc_b_bytes(NT);
  constexpr int OFF_SUM = OFF_RS + TC_ROWS * K::RS;
  constexpr int OFF_AS = OFF_SUM + NT * 16 * 4;

  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_sh;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int R0 = blockIdx.x * TC_ROWS, T0 = blockIdx.y * NT;
  const int nb = p.nb, U = p.U, n_rows = p.n_rows;

  if (warp == 0) {
    tmem_alloc(&tmem_sh, NCOLS);
    tmem_relinquish();
  }
  if (tid == 32) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_fence_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;

  // unit base and block count of each row this thread loads (rows m = i & 127)
  auto unit_of = [&](int r, size_t& base, size_t& cnt, size_t& t0) {
    const int u = r / U, ru = min(U, n_rows - u * U);
    base = (size_t)u * U * nb * K::BB;
    cnt = (size_t)ru * nb;
    t0 = (size_t)(r - u * U) * nb;  // block index of the row's block 0 inside its unit
  };

  // ---- per-thread loads of one block -----------------------------------
  // Q4_K: 4 (row, qs plane) pieces + 2 (row, scale word) pieces per thread.
  // Q6_K: 2 (row, half, sub) triples (two ql planes and one qh plane) + the
  //       row's scales (threads 0..127) and d (threads 128..255).
  constexpr int NA = T == T_Q4_K ? 4 : 6;
  struct Blk { uint4 ra[NA]; uint32_t rs[4]; uint4 rb[BV]; float ras; };
  auto load_block = [&](Blk& q, int b) {
    uint4(&ra)[NA] = q.ra;
    uint32_t(&rs)[4] = q.rs;
    uint4(&rb)[BV] = q.rb;
    float& ras = q.ras;
    if (T == T_Q4_K) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = tid + j * TC_THREADS, m = i & 127, pl = i >> 7, r = R0 + m;
        ra[j] = make_uint4(0, 0, 0, 0);
        if (r < n_rows) {
          size_t base, cnt, t0;
          unit_of(r, base, cnt, t0);
          ra[j] = __ldg(reinterpret_cast<const uint4*>(p.w + base + cnt * 16 * pl + (t0 + b) * 16));
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int i = tid + j * TC_THREADS, m = i & 127, wd = i >> 7, r = R0 + m;
        rs[j] = 0;
        if (r < n_rows) {
          size_t base, cnt, t0;
          unit_of(r, base, cnt, t0);
          // planes after qs: scales words at cnt*128, *132, *136, d|dmin at cnt*140 (wd 0..3)
          rs[j] = __ldg(reinterpret_cast<const unsigned*>(p.w + base + cnt * (128 + 4 * wd) + (t0 + b) * 4));
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int i = tid + j * TC_THREADS, m = i & 127, hs = i >> 7;  // hs = half * 2 + sub
        const int half = hs >> 1, sub = hs & 1, r = R0 + m;
        ra[3 * j] = ra[3 * j + 1] = ra[3 * j + 2] = make_uint4(0, 0, 0, 0);
        if (r < n_rows) {
          size_t base, cnt, t0;
          unit_of(r, base, cnt, t0);
          const uint8_t* blk = p.w + base + (t0 + b) * 16;
          ra[3 * j] = __ldg(reinterpret_cast<const uint4*>(blk + cnt * 16 * (half * 4 + sub)));          // ql, k&1 = 0
          ra[3 * j + 1] = __ldg(reinterpret_cast<const uint4*>(blk + cnt * 16 * (half * 4 + 2 + sub)));  // ql, k&1 = 1
          ra[3 * j + 2] = __ldg(reinterpret_cast<const uint4*>(blk + cnt * (128 + 16 * (half * 2 + sub))));  // qh
        }
      }
      const int m = tid & 127, r = R0 + m;
      rs[0] = rs[1] = rs[2] = rs[3] = 0;
      if (r < n_rows) {
        size_t base, cnt, t0;
        unit_of(r, base, cnt, t0);
        if (tid < 128) {
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.w + base + cnt * 192 + (t0 + b) * 16));
          rs[0] = v.x; rs[1] = v.y; rs[2] = v.z; rs[3] = v.w;
        } else {
          rs[0] = __ldg(reinterpret_cast<const unsigned short*>(p.w + base + cnt * 208 + (t0 + b) * 2));
        }
      }
    }
#pragma unroll
    for (int j = 0; j < BV; ++j) {
      const int i = tid + j * TC_THREADS;
      const int n = i % NT, c = i / NT;
      rb[j] = make_uint4(0, 0, 0, 0);
      if (i < NT * 16 && T0 + n < p.n_tok)
        rb[j] = __ldg(reinterpret_cast<const uint4*>(p.xq + (size_t)(T0 + n) * p.K + (size_t)b * 256 + c * 16));
    }
    ras = 0.0f;
    if (tid < NT && T0 + tid < p.n_tok) ras = __ldg(p.xs + (size_t)(T0 + tid) * nb + b);
  };

  auto store_block = [&](const Blk& q, int buf) {
    const uint4(&ra)[NA] = q.ra;
    const uint32_t(&rs)[4] = q.rs;
    const uint4(&rb)[BV] = q.rb;
    const float ras = q.ras;
    uint8_t* sb = smem + buf * BUF;
    uint8_t* a = sb;
    if (T == T_Q4_K) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = tid + j * TC_THREADS, m = i & 127, pl = i >> 7;
        uint8_t* dst = a + (m >> 3) * 2048 + (m & 7) * 16;
        const int kc = (pl >> 1) * 4 + (pl & 1);  // low nibbles: sub-block 2*(pl>>1); high: +1
        uint4 lo, hi;
        lo.x = ra[j].x & 0x0F0F0F0Fu; hi.x = (ra[j].x >> 4) & 0x0F0F0F0Fu;
        lo.y = ra[j].y & 0x0F0F0F0Fu; hi.y = (ra[j].y >> 4) & 0x0F0F0F0Fu;
        lo.z = ra[j].z & 0x0F0F0F0Fu; hi.z = (ra[j].z >> 4) & 0x0F0F0F0Fu;
        lo.w = ra[j].w & 0x0F0F0F0Fu; hi.w = (ra[j].w >> 4) & 0x0F0F0F0Fu;
        *reinterpret_cast<uint4*>(dst + kc * 128) = lo;
        *reinterpret_cast<uint4*>(dst + (kc + 2) * 128) = hi;
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int i = tid + j * TC_THREADS, m = i & 127, wd = i >> 7;
        reinterpret_cast<uint32_t*>(sb + OFF_RS + m * K::RS)[wd] = rs[j];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int i = tid + j * TC_THREADS, m = i & 127, hs = i >> 7;
        const int half = hs >> 1, sub = hs & 1;
        uint8_t* dst = a + (m >> 3) * 2048 + (m & 7) * 16;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint4 ql = ra[3 * j + (k & 1)], qh = ra[3 * j + 2];
          const int ls = 4 * (k >> 1), hsft = 2 * k;
          uint4 v;
          v.x = ((ql.x >> ls) & 0x0F0F0F0Fu) | (((qh.x >> hsft) & 0x03030303u) << 4);
          v.y = ((ql.y >> ls) & 0x0F0F0F0Fu) | (((qh.y >> hsft) & 0x03030303u) << 4);
          v.z = ((ql.z >> ls) & 0x0F0F0F0Fu) | (((qh.z >> hsft) & 0x03030303u) << 4);
          v.w = ((ql.w >> ls) & 0x0F0F0F0Fu) | (((qh.w >> hsft) & 0x03030303u) << 4);
          const int kc = half * 8 + 2 * k + sub;
          *reinterpret_cast<uint4*>(dst + kc * 128) = v;
        }
      }
      const int m = tid & 127;
      uint32_t* row = reinterpret_cast<uint32_t*>(sb + OFF_RS + m * K::RS);
      if (tid < 128) { row[0] = rs[0]; row[1] = rs[1]; row[2] = rs[2]; row[3] = rs[3]; }
      else row[4] = rs[0];
    }
    int* sums = reinterpret_cast<int*>(sb + OFF_SUM);
#pragma unroll
    for (int j = 0; j < BV; ++j) {
      const int i = tid + j * TC_THREADS;
      if (i < NT * 16) {
        const int n = i % NT, c = i / NT;
        const int off = (n >> 3) * 2048 + c * 128 + (n & 7) * 16;
        if (K::NBV == 1) {
          *reinterpret_cast<uint4*>(sb + OFF_B + off) = rb[j];
        } else {  // B0: even chunks, B1: odd chunks
          const uint4 z = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(sb + OFF_B + off) = (c & 1) ? z : rb[j];
          *reinterpret_cast<uint4*>(sb + OFF_B + tc_b_bytes(NT) + off) = (c & 1) ? rb[j] : z;
        }
        int s4 = dp4a(0x01010101u, rb[j].x, 0);
        s4 = dp4a(0x01010101u, rb[j].y, s4);
        s4 = dp4a(0x01010101u, rb[j].z, s4);
        s4 = dp4a(0x01010101u, rb[j].w, s4);
        sums[n * 16 + c] = s4;
      }
    }
    if (tid < NT) reinterpret_cast<float*>(sb + OFF_AS)[tid] = ras;
  };

  const int q4 = warp & 3, half = warp >> 2, m = q4 * 32 + lane;
  float acc[HALF];
#pragma unroll
  for (int j = 0; j < HALF; ++j) acc[j] = 0.0f;
  bool ok = true;
  int last = -1;
  auto tm = [&](int buf, int id) {  // this warp's TMEM address of accumulator id
    return tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)((buf * K::NACC + id) * NT + half * HALF);
  };

  auto fold = [&](int e) -> bool {
    const int eb = e & 1;
    const bool got = mbar_wait(&bars[eb], (unsigned)((e >> 1) & 1));
    if (!__syncthreads_and(got)) return false;
    tc_fence_after();
    const uint8_t* sb = smem + eb * BUF;
    const int* sums = reinterpret_cast<const int*>(sb + OFF_SUM);
    const float* as = reinterpret_cast<const float*>(sb + OFF_AS);
    const uint32_t* rw = reinterpret_cast<const uint32_t*>(sb + OFF_RS + m * K::RS);
    if (T == T_Q4_K) {
      const uint32_t sw[3] = {rw[0], rw[1], rw[2]};
      const float d = h2f((uint16_t)(rw[3] & 0xffff)), dmin = h2f((uint16_t)(rw[3] >> 16));
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#define SB(i) ((int)((sw[(i) >> 2] >> (8 * ((i) & 3))) & 0xffu))
        int sc, mn;
        if (j < 4) { sc = SB(j) & 63; mn = SB(j + 4) & 63; }
        else { sc = (SB(j + 4) & 0x0F) | ((SB(j - 4) >> 6) << 4); mn = (SB(j + 4) >> 4) | ((SB(j) >> 6) << 4); }
#undef SB
        uint32_t v[HALF];
        TmemLd<HALF>::run(tm(eb, j), v);
        tmem_wait_ld();
        const float dsc = __fmul_rn(d, (float)sc), dmm = __fmul_rn(dmin, (float)mn);
#pragma unroll
        for (int jj = 0; jj < HALF; ++jj) {
          const int n = half * HALF + jj;
          const int sum = sums[n * 16 + 2 * j] + sums[n * 16 + 2 * j + 1];
          const float a = __fmul_rn(dsc, __int2float_rn((int)v[jj]));
          const float bb = __fmul_rn(dmm, __int2float_rn(sum));
          acc[jj] = __fadd_rn(acc[jj], __fmul_rn(as[n], __fsub_rn(a, bb)));
        }
      }
    } else {
      const float d = h2f((uint16_t)(rw[4] & 0xffff));
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int hf = g >> 1, sub = g & 1;
        int G[HALF];
#pragma unroll
        for (int jj = 0; jj < HALF; ++jj) G[jj] = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int si = hf * 8 + sub + 2 * k;
          const int scale = (int)(int8_t)((rw[si >> 2] >> (8 * (si & 3))) & 0xffu);
          uint32_t v[HALF];
          TmemLd<HALF>::run(tm(eb, (hf * 4 + k) * 2 + sub), v);
          tmem_wait_ld();
          const int kc = hf * 8 + 2 * k + sub;
#pragma unroll
          for (int jj = 0; jj < HALF; ++jj) {
            const int n = half * HALF + jj;
            G[jj] += scale * ((int)v[jj] - 32 * sums[n * 16 + kc]);
          }
        }
#pragma unroll
        for (int jj = 0; jj < HALF; ++jj) {
          const int n = half * HALF + jj;
          const float ad = __fmul_rn(as[n], d);
          acc[jj] = __fadd_rn(acc[jj], __fmul_rn(ad, __int2float_rn(G[jj])));
        }
      }
    }
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
      const uint32_t a0 = smem_u32(smem + buf * BUF);
      const uint32_t bq = smem_u32(smem + buf * BUF + OFF_B);
      if (T == T_Q4_K) {
#pragma unroll
        for (int j = 0; j < 8; ++j)  // sub-block j: K bytes 32j .. 32j + 31
          mma_i8(tmem + (uint32_t)((buf * K::NACC + j) * NT), umma_desc(a0 + j * 256, 128, 2048),
                 umma_desc(bq + j * 256, 128, 2048), IDESC, 0u);
      } else {
#pragma unroll
        for (int c = 0; c < 8; ++c)
#pragma unroll
          for (int sub = 0; sub < 2; ++sub)
            mma_i8(tmem + (uint32_t)((buf * K::NACC + c * 2 + sub) * NT), umma_desc(a0 + c * 256, 128, 2048),
                   umma_desc(bq + sub * tc_b_bytes(NT) + c * 256, 128, 2048), IDESC, 0u);
      }
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
      for (int jj = 0; jj < HALF; ++jj) {
        const int t = T0 + half * HALF + jj;
        if (t < p.n_tok) p.out[(size_t)t * p.out_stride + r] = acc[jj];
      }
  } else {
    if (tid == 0 && p.err) atomicExch(p.err, 1);
    if (last >= 0) mbar_wait(&bars[last & 1], (unsigned)((last >> 1) & 1));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, NCOLS);
}

}  // namespace fox
