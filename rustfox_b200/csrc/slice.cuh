// Resident-slice GEMV for the ternary layer matrices of the decode step
// (sm_100a).
//
// Each CTA owns a contiguous run of whole units of the packed matrix (the
// layout of pack.cuh, with small units so the runs are even). Its first act is
// one bulk asynchronous copy (cp.async.bulk, completion counted on an
// mbarrier) of that whole run into shared memory. It then releases the next
// kernel of the stream (griddepcontrol.launch_dependents), and only after that
// waits for its own predecessor (griddepcontrol.wait). The weight stream of a
// layer therefore overlaps the previous kernel's tail, and once the
// activations are ready every weight is already on chip.
//
// Threads work in pairs. The two lanes l and l+16 of a warp split one 256
// block into two halves of 128 elements, so each lane keeps 34 (TQ1_0) or 32
// (TQ2_0) activation words in registers, not 64. A pair keeps one block
// column for the whole kernel: pair p decodes column p % nb of the rows
// p / nb, p / nb + S, ..., where S = pairs / nb. The halves' int32 sums meet
// through one shuffle. One thread per row then folds the row's block terms in
// upstream's order, exactly as the unit kernel in gemv.cuh does (upstream
// src/gemv.c:54-97, src/ternary.c:226-246). The results are bit-identical to
// it.
//
// TQ1_0 decode (upstream src/ternary.c:59-93). Byte c holds trits t_l,
// l = 0..4, with t_l + 1 = ((c * 3^l mod 256) * 3) >> 8. With
// H_l = floor(c * 3^(l+1) / 256), this is t_l + 1 = H_l - 3 H_(l-1).
// Two bytes sit in the 16-bit lanes of one register, so c * 3^(l+1)
// (at most 255 * 243 < 2^16) never carries into the next lane. A byte_perm
// gathers the four H_l of a word, and the dot product over the levels is
//   sum_l dp4a(H_l, x_l) - 3 sum_l dp4a(H_l, x_(l+1)) - sum(x).
// That is two unsigned-by-signed dp4a per level and no masking. The integer
// sum is the same as upstream's.
#pragma once

#include <algorithm>

#include "gemv.cuh"

// Phase timestamps for an instrumented build (empty here).
#ifndef FOX_SLICE_MARK
#define FOX_SLICE_MARK(k)
#endif

namespace fox {


// ---- half-block decoders ---------------------------------------------------
template <int T> struct HalfW;

// TQ1_0 half h of a block: qs[16h..16h+16) (5 levels, elements l*32 + m),
// qs[32+8h..32+8h+8) (5 levels, elements 160 + l*16 + m'), and qh bytes 2h, 2h+1
// (4 levels, elements 240 + l*4 + m''). NX activation words per half.
template <> struct HalfW<T_TQ1_0> {
  static constexpr int NX = 34;
  // activation word index (within the block's 64) of the half's i-th word
  static FOX_DEV int xword(int h, int i) {
    if (i < 20) return 8 * (i / 4) + 4 * h + (i % 4);   // level i/4, word i%4 of qs[16h..]
    if (i < 30) { const int j = i - 20; return 40 + 4 * (j / 2) + 2 * h + (j % 2); }
    return 60 + (i - 30);                                // qh levels 0..3 (masked halves)
  }
  template <int L>
  static FOX_DEV void word(uint32_t c, const uint32_t* xa, int xs, int& a1, int& a3) {
    const uint32_t lo = __byte_perm(c, 0u, 0x4240), hi = __byte_perm(c, 0u, 0x4341);
    uint32_t pl = lo, ph = hi;
#pragma unroll
    for (int l = 0; l < L; ++l) {
      pl *= 3u;
      ph *= 3u;
      const uint32_t H = __byte_perm(pl, ph, 0x7351);
      a1 = dp4a_us(H, xa[l * xs], a1);
      if (l + 1 < L) a3 = dp4a_us(H, xa[(l + 1) * xs], a3);
    }
  }
  // int32 sum over the half, without the -sum(x) offset
  static FOX_DEV int isum(const uint8_t* base, int cnt, int t, int h, const uint32_t* xa) {
    const uint4 q = *reinterpret_cast<const uint4*>(base + h * cnt * 16 + t * 16);
    const uint4 r = *reinterpret_cast<const uint4*>(base + cnt * 32 + t * 16);
    const uint32_t qh = *reinterpret_cast<const uint32_t*>(base + cnt * 48 + t * 4);
    int a1 = 0, a3 = 0;
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) word<5>(w[k], xa + k, 4, a1, a3);
    const uint32_t r0 = h ? r.z : r.x, r1 = h ? r.w : r.y;
    word<5>(r0, xa + 20, 2, a1, a3);
    word<5>(r1, xa + 21, 2, a1, a3);
    // qh: this half's two bytes; the other two zeroed so they add nothing
    word<4>(qh & (h ? 0xFFFF0000u : 0x0000FFFFu), xa + 30, 1, a1, a3);
    return a1 - 3 * a3;
  }
  static FOX_DEV float scale(const uint8_t* base, int cnt, int t) {
    return h2f(*reinterpret_cast<const uint16_t*>(base + cnt * 52 + t * 2));
  }
};

// TQ2_0 half h: qs[32h..32h+32) = planes 2h, 2h+1; element j*128 + l*32 + m is
// bits 2l..2l+1 of qs[j*32+m] (upstream src/ternary.c:177-188). One mask and
// one dp4a per four weights. TQ1_0 layer matrices are transcoded to this
// layout when a model is loaded (tq1_to_tq2_kernel), which keeps every
// integer block sum and costs a quarter of the TQ1_0 decode.
template <> struct HalfW<T_TQ2_0> {
  static constexpr int NX = 32;
  static FOX_DEV int xword(int h, int i) { return 32 * h + i; }
  static FOX_DEV int isum(const uint8_t* base, int cnt, int t, int h, const uint32_t* xa) {
    const uint4 a = *reinterpret_cast<const uint4*>(base + (2 * h) * cnt * 16 + t * 16);
    const uint4 b = *reinterpret_cast<const uint4*>(base + (2 * h + 1) * cnt * 16 + t * 16);
    const uint32_t c[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    // level l is masked in place (codes times 4^l, at most 192 per byte) and
    // summed on its own; the shifts at the end divide exactly
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int w = 0; w < 8; ++w)
#pragma unroll
      for (int l = 0; l < 4; ++l)
        acc[l] = dp4a_us(c[w] & (0x03030303u << (2 * l)), xa[l * 8 + w], acc[l]);
    return acc[0] + (acc[1] >> 2) + (acc[2] >> 4) + (acc[3] >> 6);
  }
  static FOX_DEV float scale(const uint8_t* base, int cnt, int t) {
    return h2f(*reinterpret_cast<const uint16_t*>(base + cnt * 64 + t * 2));
  }
};

// Step 5 of the slice kernels: the block terms of `rows` rows of whole
// units held in shared memory at byte offset `wofs` (unit u at wofs + u *
// ubytes), into part[(rbase + r) * rstride + col]. Pair (slot, col) takes
// rows slot, slot + S, slot + 2S, ..., two rows a pass: the two half-block
// sums are independent chains, and the pass's index work is shared. A last
// pass with no second rows (the same for the whole CTA) decodes one. Rows
// past the end are decoded from row 0 and discarded, so every lane runs the
// same straight-line code (the shuffle needs the whole warp). 32-bit shared
// memory offsets throughout.
template <typename H>
FOX_DEV void slice_terms(const unsigned char* smem, int wofs, int ubytes, int U, int nb, int rows, int S, int slot,
                         int col, int h, bool active, const uint32_t* xa, int sx, float* part, int rstride,
                         int rbase) {
  const int cnt = U * nb;
  const int ushift = __ffs(U) - 1;  // U is a power of two (2, 4 or 8)
  const int passes = (rows + 2 * S - 1) / (2 * S);
  for (int ps = 0; ps < passes; ++ps) {
    const int r0 = slot + 2 * ps * S, r1 = r0 + S;
    const bool on0 = active && r0 < rows, on1 = active && r1 < rows;
    const int q0 = on0 ? r0 : 0, q1 = on1 ? r1 : 0;
    const int ul0 = q0 >> ushift, ul1 = q1 >> ushift;
    const int t0 = (q0 - ul0 * U) * nb + col, t1 = (q1 - ul1 * U) * nb + col;
    const unsigned char* b0 = smem + wofs + ul0 * ubytes;
    const unsigned char* b1 = smem + wofs + ul1 * ubytes;
    if ((2 * ps + 1) * S < rows) {
      int v0 = H::isum(b0, cnt, t0, h, xa) - sx;
      int v1 = H::isum(b1, cnt, t1, h, xa) - sx;
      v0 += __shfl_xor_sync(0xffffffffu, v0, 16);
      v1 += __shfl_xor_sync(0xffffffffu, v1, 16);
      if (h == 0) {
        if (on0) part[(rbase + r0) * rstride + col] = __fmul_rn(H::scale(b0, cnt, t0), __int2float_rn(v0));
        if (on1) part[(rbase + r1) * rstride + col] = __fmul_rn(H::scale(b1, cnt, t1), __int2float_rn(v1));
      }
    } else {
      int v0 = H::isum(b0, cnt, t0, h, xa) - sx;
      v0 += __shfl_xor_sync(0xffffffffu, v0, 16);
      if (h == 0 && on0) part[(rbase + r0) * rstride + col] = __fmul_rn(H::scale(b0, cnt, t0), __int2float_rn(v0));
    }
  }
}

// A row's block terms added in upstream's block order, from 0.0f.
FOX_DEV float fold_row(const float* pr, int nb) {
  float acc = 0.0f;
  for (int i = 0; i < nb; ++i) acc = __fadd_rn(acc, pr[i]);
  return acc;
}

constexpr int SLICE_THREADS = 384;
// Each launch asks for at least this much shared memory, so that at most two
// CTAs of these kernels share an SM: the one finishing and the one starting.
constexpr size_t SLICE_MIN_SMEM = 96 * 1024;
constexpr size_t SLICE_MAX_SMEM = 112 * 1024;

struct SliceGeom {
  int units, per;      // units in the matrix; at most `per` per CTA
  size_t unit_bytes;   // bytes of one (full) unit
  size_t smem;         // dynamic shared memory of a launch
  size_t w_off, x_off, nw_off, xq_off, part_off, vals_off, red_off, bar_off;
};

// Shared memory plan of one launch over `grid` CTAs.
inline SliceGeom slice_geom(int type, int pro, int n_rows, int K, int U, int grid) {
  SliceGeom g;
  const int nb = K / 256;
  g.units = n_rows / U;
  g.per = (g.units + grid - 1) / grid;
  g.unit_bytes = (size_t)U * nb * block_bytes(type);
  size_t s = 0;
  g.w_off = s; s += (size_t)g.per * g.unit_bytes;
  s = (s + 15) / 16 * 16;
  // the staged floats are dead once quantised: the row terms reuse them
  const int rows = g.per * U;
  const size_t xbytes = pro != PRO_PREQ ? (size_t)K * 4 : 0;
  const size_t pbytes = (size_t)rows * (nb + 1) * 4;
  g.x_off = g.part_off = s; s += std::max(xbytes, pbytes);
  s = (s + 15) / 16 * 16;
  g.nw_off = s; if (pro_norms(pro)) s += (size_t)K * 4;
  g.xq_off = s; s += (size_t)nb * XQ_STRIDE;
  s = (s + 15) / 16 * 16;
  g.vals_off = s; s += (size_t)rows * 4;
  s = (s + 15) / 16 * 16;
  g.red_off = s; s += 32 * 8;
  g.bar_off = s; s += 16;  // two mbarriers: the weights, the norm weights
  g.smem = std::max(s, SLICE_MIN_SMEM);
  (void)type;
  return g;
}

template <int T, int PRO, int EPI>
__global__ void __launch_bounds__(SLICE_THREADS, 2) slice_kernel(const GemvParams p, const SliceGeom g) {
  using H = HalfW<T>;
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, nth = blockDim.x;
  const int K = p.K, nb = p.nb, U = p.U;
  const int u0 = blockIdx.x * g.per;
  const int nu = min(g.per, g.units - u0);
  uint8_t* sw = smem + g.w_off;
  float* xs = reinterpret_cast<float*>(smem + g.x_off);
  float* nw = reinterpret_cast<float*>(smem + g.nw_off);
  int8_t* xq = reinterpret_cast<int8_t*>(smem + g.xq_off);
  float* part = reinterpret_cast<float*>(smem + g.part_off);
  float* vals = reinterpret_cast<float*>(smem + g.vals_off);
  double* red = reinterpret_cast<double*>(smem + g.red_off);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + g.bar_off);  // [0] weights, [1] norm
  FOX_SLICE_MARK(0);

  // 1. everything constant comes in before the wait: the norm weights first
  //    (the prologue needs them before any weight, and issued after the
  //    ~100 KB run they would land last), then the CTA's run of units
  //    (contiguous in the packed matrix)
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 1);
    mbar_fence_init();
    if (pro_norms(PRO)) {
      mbar_arrive_expect_tx(bar + 1, (unsigned)(K * 4));
      bulk_g2s(nw, p.norm_w, (unsigned)(K * 4), bar + 1);
    }
    if (nu > 0) {
      const size_t total = (size_t)nu * g.unit_bytes;
      mbar_arrive_expect_tx(bar, (unsigned)total);
      const uint8_t* src = p.w + (size_t)u0 * g.unit_bytes;
      for (size_t o = 0; o < total; o += 32768)
        bulk_g2s(sw + o, src + o, (unsigned)std::min<size_t>(32768, total - o), bar);
    }
  }
  griddep_launch_dependents();
  // 2. the activations come from the previous kernel
  griddep_wait();
  __syncthreads();  // the barriers are initialised before anyone polls them
  FOX_SLICE_MARK(1);

  bool got = true;
  float am = 0.0f;
  if (PRO != PRO_PREQ) {
    const uint32_t fep = PRO == PRO_NFOLD ? tp_epoch(p.pos, p.f_phase) : 0u;
    bool fok = true;
    double ss = 0.0;
    for (int i = tid * 4; i < K; i += nth * 4) {
      const float4 v = PRO == PRO_NFOLD ? nfold_x4(p, i, K, fep, &fok) : *reinterpret_cast<const float4*>(p.x + i);
      if (PRO == PRO_NFOLD && blockIdx.x == 0) *reinterpret_cast<float4*>(p.f_out + i) = v;
      if (pro_norms(PRO))
        ss = ss + (double)v.x * (double)v.x + (double)v.y * (double)v.y +
             (double)v.z * (double)v.z + (double)v.w * (double)v.w;
      else
        am = absmax_acc(absmax_acc(absmax_acc(absmax_acc(am, v.x), v.y), v.z), v.w);
      *reinterpret_cast<float4*>(xs + i) = v;
    }
    FOX_SLICE_MARK(2);
    if (pro_norms(PRO)) {
      const double sum = block_reduce<double>(ss, red, OpAddD(), 0.0);
      FOX_SLICE_MARK(3);
      const float scale = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)K), (double)p.eps)));
      FOX_SLICE_MARK(4);
      got = mbar_wait(bar + 1, 0);
      FOX_SLICE_MARK(5);
      // normalise (x * scale * w, upstream src/ops.c:7-22) and take the absmax
      // in the same pass
      for (int i = tid * 4; i < K; i += nth * 4) {
        float4 v = *reinterpret_cast<float4*>(xs + i);
        const float4 w = *reinterpret_cast<const float4*>(nw + i);
        v.x = __fmul_rn(__fmul_rn(v.x, scale), w.x);
        v.y = __fmul_rn(__fmul_rn(v.y, scale), w.y);
        v.z = __fmul_rn(__fmul_rn(v.z, scale), w.z);
        v.w = __fmul_rn(__fmul_rn(v.w, scale), w.w);
        *reinterpret_cast<float4*>(xs + i) = v;
        am = absmax_acc(absmax_acc(absmax_acc(absmax_acc(am, v.x), v.y), v.z), v.w);
      }
    }
  }
  float act_scale;
  if (PRO == PRO_PREQ) {
    act_scale = p.xq_scale[0];
    for (int i = tid * 16; i < K; i += nth * 16)
      *reinterpret_cast<uint4*>(xq + (i >> 8) * XQ_STRIDE + (i & 255)) =
          *reinterpret_cast<const uint4*>(p.xq + i);
  } else {
    // upstream src/gemv.c:11-42: one absmax over the whole vector (over
    // every shard's slice: given under PRO_GSCALE, traded under PRO_XAMAX)
    FOX_SLICE_MARK(6);
    float amax;
    if (PRO == PRO_GSCALE) {
      amax = p.xq_scale[0];
    } else {
      amax = block_reduce<float>(am, (float*)red, OpMax(), 0.0f);
      if (PRO == PRO_XAMAX) amax = x_trade_amax(p, amax);
    }
    FOX_SLICE_MARK(7);
    const bool nz = amax > 0.0f;
    const float inv = nz ? __fdiv_rn(127.0f, amax) : 0.0f;
    act_scale = nz ? __fdiv_rn(amax, 127.0f) : 0.0f;
    for (int i = tid * 4; i < K; i += nth * 4) {
      const float4 v = *reinterpret_cast<const float4*>(xs + i);
      *reinterpret_cast<uint32_t*>(xq + (i >> 8) * XQ_STRIDE + (i & 255)) =
          pack4(quant1(v.x, inv), quant1(v.y, inv), quant1(v.z, inv), quant1(v.w, inv));
    }
  }
  __syncthreads();
  FOX_SLICE_MARK(8);

  // 3. this lane's half-block activations (fixed column for the whole kernel)
  const int lane = tid & 31, h = lane >> 4;
  const int pair = (tid >> 5) * 16 + (lane & 15);
  const int S = (nth >> 1) / nb;               // row slots
  const bool active = pair < S * nb;
  const int col = active ? pair % nb : 0, slot = active ? pair / nb : 0;
  uint32_t xa[H::NX];
  int sx = 0;
  {
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(xq + col * XQ_STRIDE);
    if (T == T_TQ2_0) {  // the half's 32 words are contiguous
      const uint4* x4 = reinterpret_cast<const uint4*>(xw + 32 * h);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 v = x4[i];
        xa[4 * i] = v.x; xa[4 * i + 1] = v.y; xa[4 * i + 2] = v.z; xa[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < H::NX; ++i) xa[i] = xw[H::xword(h, i)];
    }
    int s4[4] = {0, 0, 0, 0};
    if (T == T_TQ1_0) {
#pragma unroll
      for (int i = 0; i < 30; ++i) s4[i & 3] = dp4a(0x01010101u, xa[i], s4[i & 3]);
      // qh words: only this half's two bytes
      const uint32_t m = h ? 0x01010000u : 0x00000101u;
#pragma unroll
      for (int i = 30; i < 34; ++i) s4[i & 3] = dp4a(m, xa[i], s4[i & 3]);
    } else {
#pragma unroll
      for (int i = 0; i < H::NX; ++i) s4[i & 3] = dp4a(0x01010101u, xa[i], s4[i & 3]);
    }
    sx = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  }

  FOX_SLICE_MARK(9);
  // 4. weights on chip; every thread polls, the CTA leaves together if any
  //    wait gave up
  got = got && (nu <= 0 || mbar_wait(bar, 0));
  if (!__syncthreads_and(got)) {
    if (tid == 0 && p.err) atomicExch(p.err, 1);
    // give copies still in flight a second bounded wait before the shared
    // memory is released
    if (tid == 0) {
      mbar_wait(bar, 0);
      if (pro_norms(PRO)) mbar_wait(bar + 1, 0);
    }
    __syncthreads();
    // still counted, so the completion count is rearmed for the next
    // exchange; the error word marks this step's terms as unusable
    if (EPI == EPI_TERMS && p.x_count) x_signal_ready(p);
    return;
  }

  FOX_SLICE_MARK(10);
  // 5. block terms: pair (slot, col) takes rows slot, slot + S, ...
  const int rows = nu * U;
  const int rstride = nb + 1;
  slice_terms<H>(smem, (int)g.w_off, (int)g.unit_bytes, U, nb, rows, S, slot, col, h, active, xa, sx, part,
                 rstride, 0);
  __syncthreads();
  FOX_SLICE_MARK(11);

  // 6. rows in upstream's order, then the epilogue (EPI_TERMS: the block
  //    terms themselves, folded by the exchange's fold)
  const int row0 = u0 * U;
  if (EPI == EPI_TERMS)
    for (int i = tid; i < rows * nb; i += nth) {
      const int r = i / nb, c = i - r * nb;
      p.out[(size_t)(row0 + r) * p.terms_stride + c] = part[r * rstride + c];
    }
  for (int r = tid; r < rows && EPI != EPI_TERMS; r += nth) {
    const float* pr = part + r * rstride;
    const float acc = fold_row(pr, nb);
    const float v = __fmul_rn(acc, act_scale);
    if (EPI == EPI_STORE) p.out[row0 + r] = v;
    if (EPI == EPI_ADD) p.out[row0 + r] = __fadd_rn(p.out[row0 + r], v);
    if (EPI == EPI_XSUM) xsum_store(p, row0 + r, v, tp_epoch(p.pos, p.x_phase));
    if (EPI == EPI_QKV || EPI == EPI_SWIGLU) vals[r] = v;
  }
  if (EPI == EPI_QKV || EPI == EPI_SWIGLU) __syncthreads();
  if (EPI == EPI_QKV) {
    const int P = *p.pos;
    for (int r = tid; r < rows; r += nth) {
      const int rg = p.row_base + row0 + r;
      const float mine = vals[r];
      if (rg < p.nq + p.nkv) {
        const float other = vals[r ^ 1];
        const int rr = rg < p.nq ? rg : rg - p.nq;
        const int i = (rr % p.hd) >> 1;
        const float c = p.rope_cos[(size_t)P * (p.hd >> 1) + i];
        const float s = p.rope_sin[(size_t)P * (p.hd >> 1) + i];
        const bool odd = r & 1;
        const float x0 = odd ? other : mine, x1 = odd ? mine : other;
        const float o = odd ? __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c))
                            : __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        if (rg < p.nq) {
          p.out[rg] = o;
        } else {
          const size_t idx = kv_row(p.kv_table, p.n_ctx, p.nkv / p.hd, rr / p.hd, P) * p.hd + rr % p.hd;
          if (p.kv_f16) reinterpret_cast<__half*>(p.kcache)[idx] = __float2half_rn(o);
          else reinterpret_cast<float*>(p.kcache)[idx] = o;
        }
      } else {
        const int rr = rg - p.nq - p.nkv;
        const size_t idx = kv_row(p.kv_table, p.n_ctx, p.nkv / p.hd, rr / p.hd, P) * p.hd + rr % p.hd;
        if (p.kv_f16) reinterpret_cast<__half*>(p.vcache)[idx] = __float2half_rn(mine);
        else reinterpret_cast<float*>(p.vcache)[idx] = mine;
      }
    }
  }
  if (EPI == EPI_SWIGLU) {
    const int hu = U >> 1;
    for (int k = tid; k < nu * hu; k += nth) {
      const int ul = k / hu, i = k - ul * hu;
      const float gt = vals[ul * U + i], up = vals[ul * U + hu + i];
      p.out[(u0 + ul) * hu + i] = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf_up(-gt))), up);
    }
  }
  FOX_SLICE_MARK(12);
  if (EPI == EPI_TERMS && p.x_count) x_signal_ready(p);
}

// ---------------------------------------------------------------------------
// Streaming slice kernel: a ternary layer matrix larger than the shared
// memory of the grid (the 27B layer matrices: up to 57 MB against 148 x
// 224 KB). One CTA per SM owns a contiguous run of units, as above, and
// takes it in chunks through a ring of nbuf shared-memory buffers (one
// mbarrier each): chunks 0..nbuf-1 are copied before griddepcontrol.wait,
// and chunk c + nbuf is issued into the buffer chunk c has just freed, so
// nbuf - 1 chunks (about 100 KB per SM) are in flight while one is decoded
// by the CTA's 24 warps.
// The block terms of every chunk are parked for the whole run and folded
// once after the last chunk (a per-chunk fold would leave most warps idle
// at a barrier once per chunk). Decode, fold order and epilogues are the
// resident kernel's, so the rows are bit-identical to it. An activation vector longer than SLICE_STAGE_X
// bytes (the 21504-wide down input) is read from global memory (L2) in each
// prologue pass rather than staged.
constexpr int STREAM_THREADS = 768;  // one CTA per SM: 24 warps decode each chunk
constexpr size_t STREAM_MAX_SMEM = 200 * 1024;
constexpr size_t STREAM_CHUNK_BYTES = 48 * 1024;
constexpr size_t SLICE_STAGE_X = 24 * 1024;
constexpr int STREAM_MAX_BUF = 8;

struct StreamGeom {
  int units, per;      // units in the matrix; at most `per` per CTA
  int chunk, nch;      // units per chunk, chunks per CTA
  int nbuf;            // chunk buffers
  int stage_x;         // the activation vector is staged in shared memory
  size_t unit_bytes, chunk_bytes;
  size_t smem;
  size_t w_off, x_off, nw_off, xq_off, part_off, vals_off, red_off, bar_off;
};

// Plan over `grid` CTAs; nbuf 0 when not even two one-unit buffers fit.
inline StreamGeom stream_geom(int type, int pro, int n_rows, int K, int U, int grid) {
  StreamGeom g;
  const int nb = K / 256;
  g.units = n_rows / U;
  g.per = (g.units + grid - 1) / grid;
  g.unit_bytes = (size_t)U * nb * block_bytes(type);
  // about STREAM_CHUNK_BYTES per chunk, rounded to whole passes of the
  // (SLICE_THREADS / 2) / nb row slots where that keeps it near the target
  int chunk = (int)std::max<size_t>(1, std::min<size_t>((size_t)g.per, STREAM_CHUNK_BYTES / g.unit_bytes));
  const int slots = (STREAM_THREADS / 2) / nb;
  for (int c = chunk; c >= (chunk * 3) / 4 && c >= 1; --c)
    if ((c * U) % slots == 0) { chunk = c; break; }
  g.chunk = chunk;
  g.nch = (g.per + g.chunk - 1) / g.chunk;
  g.chunk_bytes = (g.chunk * g.unit_bytes + 15) / 16 * 16;
  g.stage_x = pro != PRO_PREQ && (size_t)K * 4 <= SLICE_STAGE_X ? 1 : 0;
  const int rows = g.per * U;  // the row terms of the whole run wait for one fold
  size_t s = 0;
  const size_t xbytes = g.stage_x ? (size_t)K * 4 : 0;
  const size_t pbytes = (size_t)rows * (nb + 1) * 4;
  g.x_off = g.part_off = s; s += std::max(xbytes, pbytes);
  s = (s + 15) / 16 * 16;
  g.nw_off = s; if (pro_norms(pro)) s += (size_t)K * 4;
  g.xq_off = s; s += (size_t)nb * XQ_STRIDE;
  s = (s + 15) / 16 * 16;
  g.vals_off = s; s += (size_t)rows * 4;
  s = (s + 15) / 16 * 16;
  g.red_off = s; s += 32 * 8;
  g.bar_off = s; s += 8 * (1 + STREAM_MAX_BUF);  // the norm weights, then one per buffer
  s = (s + 127) / 128 * 128;
  g.w_off = s;
  const size_t room = STREAM_MAX_SMEM > s ? STREAM_MAX_SMEM - s : 0;
  g.nbuf = (int)std::min<size_t>(STREAM_MAX_BUF, std::min<size_t>((size_t)g.nch, room / g.chunk_bytes));
  if (g.nch > 1 && g.nbuf < 2) g.nbuf = 0;
  if (g.nch == 1 && g.nbuf < 1) g.nbuf = 0;
  g.smem = s + (size_t)g.nbuf * g.chunk_bytes;
  (void)type;
  return g;
}

template <int T, int PRO, int EPI>
__global__ void __launch_bounds__(STREAM_THREADS, 1) stream_kernel(const GemvParams p, const StreamGeom g) {
  using H = HalfW<T>;
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, nth = blockDim.x;
  const int K = p.K, nb = p.nb, U = p.U;
  const int u0 = blockIdx.x * g.per;
  const int nu = min(g.per, g.units - u0);
  uint8_t* sw = smem + g.w_off;  // nbuf chunk buffers of g.chunk_bytes
  float* xs = reinterpret_cast<float*>(smem + g.x_off);
  float* nw = reinterpret_cast<float*>(smem + g.nw_off);
  int8_t* xq = reinterpret_cast<int8_t*>(smem + g.xq_off);
  float* part = reinterpret_cast<float*>(smem + g.part_off);
  float* vals = reinterpret_cast<float*>(smem + g.vals_off);
  double* red = reinterpret_cast<double*>(smem + g.red_off);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + g.bar_off);  // [0] norm, [1 + b] buffer b

  // chunk c of this CTA's run: units [c * chunk, min(nu, (c + 1) * chunk))
  auto chunk_units = [&](int c) { return min(g.chunk, nu - c * g.chunk); };
  auto issue = [&](int c) {
    const int cu = chunk_units(c);
    if (cu <= 0) return;
    uint64_t* b = bar + 1 + c % g.nbuf;
    uint8_t* dst = sw + (size_t)(c % g.nbuf) * g.chunk_bytes;
    const size_t total = (size_t)cu * g.unit_bytes;
    mbar_arrive_expect_tx(b, (unsigned)total);
    const uint8_t* src = p.w + (size_t)(u0 + c * g.chunk) * g.unit_bytes;
    for (size_t o = 0; o < total; o += 32768)
      bulk_g2s(dst + o, src + o, (unsigned)std::min<size_t>(32768, total - o), b);
  };

  // 1. everything constant comes in before the wait: the norm weights
  //    first, then the CTA's first nbuf chunks
  if (tid == 0) {
    for (int b = 0; b <= g.nbuf; ++b) mbar_init(bar + b, 1);
    mbar_fence_init();
    if (pro_norms(PRO)) {
      mbar_arrive_expect_tx(bar, (unsigned)(K * 4));
      bulk_g2s(nw, p.norm_w, (unsigned)(K * 4), bar);
    }
    for (int c = 0; c < min(g.nbuf, g.nch); ++c) issue(c);
  }
  griddep_launch_dependents();
  // 2. the activations come from the previous kernel
  griddep_wait();
  __syncthreads();  // the barriers are initialised before anyone polls them

  bool got = true;
  float am = 0.0f;
  float norm_scale = 1.0f;
  const uint32_t fep = PRO == PRO_NFOLD ? tp_epoch(p.pos, p.f_phase) : 0u;
  bool fok = true;
  // the input, completed from the ranks' row sums under PRO_NFOLD
  auto load4 = [&](int i) -> float4 {
    if (PRO == PRO_NFOLD) return nfold_x4(p, i, K, fep, &fok);
    return *reinterpret_cast<const float4*>(p.x + i);
  };
  auto norm4 = [&](float4 v, int i) -> float4 {
    const float4 w = *reinterpret_cast<const float4*>(nw + i);
    v.x = __fmul_rn(__fmul_rn(v.x, norm_scale), w.x);
    v.y = __fmul_rn(__fmul_rn(v.y, norm_scale), w.y);
    v.z = __fmul_rn(__fmul_rn(v.z, norm_scale), w.z);
    v.w = __fmul_rn(__fmul_rn(v.w, norm_scale), w.w);
    return v;
  };
  // the prologue's value of element i..i+3 after the first pass: staged, or
  // recomputed from global memory (the same operations, the same values)
  auto value4 = [&](int i) -> float4 {
    if (g.stage_x) return *reinterpret_cast<const float4*>(xs + i);
    const float4 v = load4(i);
    return pro_norms(PRO) ? norm4(v, i) : v;
  };
  if (PRO != PRO_PREQ) {
    double ss = 0.0;
    for (int i = tid * 4; i < K; i += nth * 4) {
      const float4 v = load4(i);
      if (PRO == PRO_NFOLD && blockIdx.x == 0) *reinterpret_cast<float4*>(p.f_out + i) = v;
      if (pro_norms(PRO))
        ss = ss + (double)v.x * (double)v.x + (double)v.y * (double)v.y +
             (double)v.z * (double)v.z + (double)v.w * (double)v.w;
      else
        am = absmax_acc(absmax_acc(absmax_acc(absmax_acc(am, v.x), v.y), v.z), v.w);
      if (g.stage_x) *reinterpret_cast<float4*>(xs + i) = v;
    }
    if (pro_norms(PRO)) {
      const double sum = block_reduce<double>(ss, red, OpAddD(), 0.0);
      norm_scale = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)K), (double)p.eps)));
      got = mbar_wait(bar, 0);
      // normalise (x * scale * w, upstream src/ops.c:7-22) and take the absmax
      // in the same pass
      for (int i = tid * 4; i < K; i += nth * 4) {
        const float4 v = norm4(g.stage_x ? *reinterpret_cast<const float4*>(xs + i) : load4(i), i);
        if (g.stage_x) *reinterpret_cast<float4*>(xs + i) = v;
        am = absmax_acc(absmax_acc(absmax_acc(absmax_acc(am, v.x), v.y), v.z), v.w);
      }
    }
  }
  float act_scale;
  if (PRO == PRO_PREQ) {
    act_scale = p.xq_scale[0];
    for (int i = tid * 16; i < K; i += nth * 16)
      *reinterpret_cast<uint4*>(xq + (i >> 8) * XQ_STRIDE + (i & 255)) =
          *reinterpret_cast<const uint4*>(p.xq + i);
  } else {
    // upstream src/gemv.c:11-42: one absmax over the whole vector (over
    // every shard's slice: given under PRO_GSCALE, traded under PRO_XAMAX)
    float amax;
    if (PRO == PRO_GSCALE) {
      amax = p.xq_scale[0];
    } else {
      amax = block_reduce<float>(am, (float*)red, OpMax(), 0.0f);
      if (PRO == PRO_XAMAX) amax = x_trade_amax(p, amax);
    }
    const bool nz = amax > 0.0f;
    const float inv = nz ? __fdiv_rn(127.0f, amax) : 0.0f;
    act_scale = nz ? __fdiv_rn(amax, 127.0f) : 0.0f;
    for (int i = tid * 4; i < K; i += nth * 4) {
      const float4 v = value4(i);
      *reinterpret_cast<uint32_t*>(xq + (i >> 8) * XQ_STRIDE + (i & 255)) =
          pack4(quant1(v.x, inv), quant1(v.y, inv), quant1(v.z, inv), quant1(v.w, inv));
    }
  }
  __syncthreads();

  // 3. this lane's half-block activations (fixed column for the whole kernel)
  const int lane = tid & 31, h = lane >> 4;
  const int pair = (tid >> 5) * 16 + (lane & 15);
  const int S = (nth >> 1) / nb;               // row slots
  const bool active = pair < S * nb;
  const int col = active ? pair % nb : 0, slot = active ? pair / nb : 0;
  uint32_t xa[H::NX];
  int sx = 0;
  {
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(xq + col * XQ_STRIDE);
    if (T == T_TQ2_0) {  // the half's 32 words are contiguous
      const uint4* x4 = reinterpret_cast<const uint4*>(xw + 32 * h);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 v = x4[i];
        xa[4 * i] = v.x; xa[4 * i + 1] = v.y; xa[4 * i + 2] = v.z; xa[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < H::NX; ++i) xa[i] = xw[H::xword(h, i)];
    }
    int s4[4] = {0, 0, 0, 0};
    if (T == T_TQ1_0) {
#pragma unroll
      for (int i = 0; i < 30; ++i) s4[i & 3] = dp4a(0x01010101u, xa[i], s4[i & 3]);
      // qh words: only this half's two bytes
      const uint32_t m = h ? 0x01010000u : 0x00000101u;
#pragma unroll
      for (int i = 30; i < 34; ++i) s4[i & 3] = dp4a(m, xa[i], s4[i & 3]);
    } else {
#pragma unroll
      for (int i = 0; i < H::NX; ++i) s4[i & 3] = dp4a(0x01010101u, xa[i], s4[i & 3]);
    }
    sx = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  }

  const int rstride = nb + 1;
  for (int c = 0; c < g.nch; ++c) {
    const int cu = chunk_units(c);
    if (cu <= 0) break;
    // 4. this chunk's weights on chip: warp 0 polls (the other 23 warps
    //    wait at the barrier instead of spending issue slots on polls), the
    //    barrier passes the completed phase on to the CTA; the CTA leaves
    //    together if any wait gave up
    if (tid < 32) got = got && mbar_wait(bar + 1 + c % g.nbuf, (c / g.nbuf) & 1);
    if (!__syncthreads_and(got)) {
      if (tid == 0 && p.err) atomicExch(p.err, 1);
      // give copies still in flight a second bounded wait before the shared
      // memory is released
      if (tid == 0) {
        for (int j = c; j < min(g.nch, c + g.nbuf); ++j)
          if (chunk_units(j) > 0) mbar_wait(bar + 1 + j % g.nbuf, (j / g.nbuf) & 1);
        if (pro_norms(PRO)) mbar_wait(bar, 0);
      }
      __syncthreads();
      // still counted, so the completion count is rearmed for the next
      // exchange; the error word marks this step's sums as unusable
      if (EPI == EPI_TERMS && p.x_count) x_signal_ready(p);
      return;
    }
    const int wofs = (int)(g.w_off + (size_t)(c % g.nbuf) * g.chunk_bytes);  // this chunk's buffer

    // 5. block terms of the chunk's rows, parked with the run's other rows
    //    (folded once, after the last chunk): pair (slot, col) takes rows
    //    slot, slot + S, ...
    const int rows = cu * U;
    const int rbase = c * g.chunk * U;  // the chunk's first row within the run
    slice_terms<H>(smem, wofs, (int)g.unit_bytes, U, nb, rows, S, slot, col, h, active, xa, sx, part, rstride,
                   rbase);
    __syncthreads();
    // the buffer is free: chunk c + nbuf streams in behind the others
    if (tid == 0 && c + g.nbuf < g.nch) issue(c + g.nbuf);
  }
  // a CTA without units still waits out its norm-weight copy when the first
  // wait gave up, before its shared memory is released
  if (nu <= 0 && !__syncthreads_and(got)) {
    if (tid == 0) {
      if (p.err) atomicExch(p.err, 1);
      if (pro_norms(PRO)) mbar_wait(bar, 0);
    }
    __syncthreads();
  }

  // 6. rows in upstream's order, then the epilogue (EPI_TERMS: the block
  //    terms themselves, folded by the exchange's fold)
  const int rows = max(nu, 0) * U;
  const int row0 = u0 * U;
  if (EPI == EPI_TERMS)
    for (int i = tid; i < rows * nb; i += nth) {
      const int r = i / nb, cc = i - r * nb;
      p.out[(size_t)(row0 + r) * p.terms_stride + cc] = part[r * rstride + cc];
    }
  for (int r = tid; r < rows && EPI != EPI_TERMS; r += nth) {
    const float* pr = part + r * rstride;
    const float acc = fold_row(pr, nb);
    const float v = __fmul_rn(acc, act_scale);
    if (EPI == EPI_STORE) p.out[row0 + r] = v;
    if (EPI == EPI_ADD) p.out[row0 + r] = __fadd_rn(p.out[row0 + r], v);
    if (EPI == EPI_XSUM) xsum_store(p, row0 + r, v, tp_epoch(p.pos, p.x_phase));
    if (EPI == EPI_QKV || EPI == EPI_SWIGLU) vals[r] = v;
  }
  if (EPI == EPI_QKV || EPI == EPI_SWIGLU) __syncthreads();
  if (EPI == EPI_QKV) {
    const int P = *p.pos;
    for (int r = tid; r < rows; r += nth) {
      const int rg = p.row_base + row0 + r;
      const float mine = vals[r];
      if (rg < p.nq + p.nkv) {
        const float other = vals[r ^ 1];
        const int rr = rg < p.nq ? rg : rg - p.nq;
        const int i = (rr % p.hd) >> 1;
        const float cs = p.rope_cos[(size_t)P * (p.hd >> 1) + i];
        const float sn = p.rope_sin[(size_t)P * (p.hd >> 1) + i];
        const bool odd = r & 1;
        const float x0 = odd ? other : mine, x1 = odd ? mine : other;
        const float o = odd ? __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs))
                            : __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        if (rg < p.nq) {
          p.out[rg] = o;
        } else {
          const size_t idx = kv_row(p.kv_table, p.n_ctx, p.nkv / p.hd, rr / p.hd, P) * p.hd + rr % p.hd;
          if (p.kv_f16) reinterpret_cast<__half*>(p.kcache)[idx] = __float2half_rn(o);
          else reinterpret_cast<float*>(p.kcache)[idx] = o;
        }
      } else {
        const int rr = rg - p.nq - p.nkv;
        const size_t idx = kv_row(p.kv_table, p.n_ctx, p.nkv / p.hd, rr / p.hd, P) * p.hd + rr % p.hd;
        if (p.kv_f16) reinterpret_cast<__half*>(p.vcache)[idx] = __float2half_rn(mine);
        else reinterpret_cast<float*>(p.vcache)[idx] = mine;
      }
    }
  }
  if (EPI == EPI_SWIGLU) {
    const int hu = U >> 1;
    for (int k = tid; k < max(nu, 0) * hu; k += nth) {
      const int ul = k / hu, i = k - ul * hu;
      const float gt = vals[ul * U + i], up = vals[ul * U + hu + i];
      p.out[(u0 + ul) * hu + i] = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf_up(-gt))), up);
    }
  }
  if (EPI == EPI_TERMS && p.x_count) x_signal_ready(p);
}

}  // namespace fox
