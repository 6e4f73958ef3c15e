// libfoxcuda: the C ABI (include/foxcuda.h), the HBM weight store, the decode
// context and its CUDA graphs.
#include <cuda_runtime.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

#include "../../include/foxcuda.h"
#include "common.cuh"
#include "gemv.cuh"
#include "ops.cuh"
#include "pack.cuh"
#include "slice.cuh"
#include "rows.cuh"
#include "tc.cuh"
#include "tc_kquant.cuh"
#include "prefill.cuh"
#include "p2p.cuh"
#include "attn.cuh"
#include "synthgen.cuh"

using namespace fox;

// ---------------------------------------------------------------------------
// errors: thread-local message, status codes of upstream fox_status

static thread_local char g_err[512];

static foxcuda_status fail(foxcuda_status st, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return st;
}

static foxcuda_status cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorMemoryAllocation ? FOXCUDA_ERR_NOMEM : FOXCUDA_ERR_INTERNAL,
              "%s: %s", what, cudaGetErrorString(e));
}

#define CK(call, what)                                   \
  do {                                                   \
    cudaError_t e_ = (call);                             \
    if (e_ != cudaSuccess) return cuda_fail(e_, what);   \
  } while (0)

extern "C" const char* foxcuda_last_error(void) { return g_err[0] ? g_err : "no error recorded"; }
extern "C" const char* foxcuda_version(void) { return "foxcuda 0.1.0 (sm_100a)"; }

static int sm_count(int dev) {
  static int cached[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

static int current_sms() {
  int d = 0;
  cudaGetDevice(&d);
  return sm_count(d);
}

// The dynamic shared-memory opt-in is a property of a kernel on one device,
// so each launcher keeps its high-water mark per device (`marks` has one
// slot per device ordinal). The attribute only ever rises, under a lock, so
// two threads cannot leave it below a mark that another thread relies on.
constexpr int kMaxDevices = 64;
static std::mutex g_smem_mu;

template <typename K>
static cudaError_t opt_in_smem(K kern, size_t smem, size_t* marks) {
  if (smem <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_smem_mu);
  if (smem <= marks[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  marks[dev] = smem;
  return cudaSuccess;
}

extern "C" foxcuda_status foxcuda_init(int device) {
  int n = 0;
  CK(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
  if (device < 0 || device >= n) return fail(FOXCUDA_ERR_ARG, "init: device %d of %d", device, n);
  CK(cudaSetDevice(device), "cudaSetDevice");
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "init: %s is sm_%d%d; this build is sm_100a only",
                prop.name, prop.major, prop.minor);
  return FOXCUDA_OK;
}

static bool type_gemv_ok(int t) {
  return t == T_TQ1_0 || t == T_TQ2_0 || t == T_Q4_K || t == T_Q6_K || t == T_Q8_0;
}

static size_t row_bytes(int t, size_t n_cols) {
  const int be = block_elems(t);
  if (n_cols % be) return 0;
  return n_cols / be * block_bytes(t);
}

// ---------------------------------------------------------------------------
// GEMV launch

template <int T, int PRO, int EPI>
static cudaError_t launch_gemv_t(const GemvParams& p, cudaStream_t s) {
  auto kern = gemv_kernel<T, PRO, EPI>;
  const int threads = (p.U * p.nb + 31) / 32 * 32;
  const size_t smem = gemv_smem_bytes(T, PRO, p.K, p.U, p.nb);
  static size_t marks[kMaxDevices] = {};  // per instantiation
  cudaError_t e = opt_in_smem(kern, smem, marks);
  if (e != cudaSuccess) return e;
  int occ = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem);
  if (e != cudaSuccess) return e;
  if (occ < 1) return cudaErrorInvalidConfiguration;
  const int units = (p.n_rows + p.U - 1) / p.U;
  const int grid = std::min(units, occ * current_sms());
  kern<<<grid, threads, smem, s>>>(p);
  return cudaGetLastError();
}

template <int T>
static cudaError_t launch_gemv_pe(int pro, int epi, const GemvParams& p, cudaStream_t s) {
  if (pro == PRO_VEC && epi == EPI_STORE) return launch_gemv_t<T, PRO_VEC, EPI_STORE>(p, s);
  if (pro == PRO_VEC && epi == EPI_ADD) return launch_gemv_t<T, PRO_VEC, EPI_ADD>(p, s);
  if (pro == PRO_NORM && epi == EPI_STORE) return launch_gemv_t<T, PRO_NORM, EPI_STORE>(p, s);
  if (pro == PRO_NORM && epi == EPI_QKV) return launch_gemv_t<T, PRO_NORM, EPI_QKV>(p, s);
  if (pro == PRO_NORM && epi == EPI_SWIGLU) return launch_gemv_t<T, PRO_NORM, EPI_SWIGLU>(p, s);
  if constexpr (T != T_Q8_0)
    if (pro == PRO_PREQ && epi == EPI_STORE) return launch_gemv_t<T, PRO_PREQ, EPI_STORE>(p, s);
  return cudaErrorInvalidValue;
}

static cudaError_t launch_gemv(int type, int pro, int epi, const GemvParams& p, cudaStream_t s) {
  switch (type) {
    case T_TQ1_0: return launch_gemv_pe<T_TQ1_0>(pro, epi, p, s);
    case T_TQ2_0: return launch_gemv_pe<T_TQ2_0>(pro, epi, p, s);
    case T_Q4_K: return launch_gemv_pe<T_Q4_K>(pro, epi, p, s);
    case T_Q6_K: return launch_gemv_pe<T_Q6_K>(pro, epi, p, s);
    case T_Q8_0: return launch_gemv_pe<T_Q8_0>(pro, epi, p, s);
    default: return cudaErrorInvalidValue;
  }
}

// Ring mode (gemv.cuh): about RING_BYTES of a CTA's units in flight.
constexpr size_t RING_BYTES = 96 * 1024;

template <int T, int PRO, int EPI>
static cudaError_t launch_ring_t(GemvParams p, cudaStream_t s) {
  auto kern = gemv_kernel<T, PRO, EPI, true>;
  const int threads = (p.U * p.nb + 31) / 32 * 32;
  const size_t unit = (size_t)p.U * p.nb * block_bytes(T);
  if (unit % 16) return launch_gemv_t<T, PRO, EPI>(p, s);  // not bulk-copyable
  const size_t base = (gemv_smem_bytes(T, PRO, p.K, p.U, p.nb) + 15) / 16 * 16;
  const int R = (int)std::max<size_t>(2, std::min<size_t>(8, RING_BYTES / unit));
  const size_t smem = base + (size_t)R * unit + (size_t)R * 8;
  static size_t marks[kMaxDevices] = {};  // per instantiation
  cudaError_t e = opt_in_smem(kern, smem, marks);
  if (e != cudaSuccess) return e;
  int occ = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem);
  if (e != cudaSuccess) return e;
  if (occ < 1) return cudaErrorInvalidConfiguration;
  const int units = (p.n_rows + p.U - 1) / p.U;
  const int grid = std::min(units, occ * current_sms());
  p.ring_slots = R;
  p.slot_bytes = (int)unit;
  p.ring_off = (int)base;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int T>
static cudaError_t launch_ring_pe(int pro, int epi, const GemvParams& p, cudaStream_t s) {
  if (pro == PRO_VEC && epi == EPI_STORE) return launch_ring_t<T, PRO_VEC, EPI_STORE>(p, s);
  if (pro == PRO_VEC && epi == EPI_ADD) return launch_ring_t<T, PRO_VEC, EPI_ADD>(p, s);
  if (pro == PRO_NORM && epi == EPI_STORE) return launch_ring_t<T, PRO_NORM, EPI_STORE>(p, s);
  if (pro == PRO_NORM && epi == EPI_QKV) return launch_ring_t<T, PRO_NORM, EPI_QKV>(p, s);
  if (pro == PRO_NORM && epi == EPI_SWIGLU) return launch_ring_t<T, PRO_NORM, EPI_SWIGLU>(p, s);
  // tensor-parallel sums exchange (p2p.cuh): the consumers that complete
  // the residual, the row-parallel producers
  if (pro == PRO_NFOLD && epi == EPI_QKV) return launch_ring_t<T, PRO_NFOLD, EPI_QKV>(p, s);
  if (pro == PRO_NFOLD && epi == EPI_SWIGLU) return launch_ring_t<T, PRO_NFOLD, EPI_SWIGLU>(p, s);
  if constexpr (T == T_TQ1_0 || T == T_TQ2_0) {
    if (pro == PRO_XAMAX && epi == EPI_XSUM) return launch_ring_t<T, PRO_XAMAX, EPI_XSUM>(p, s);
  } else if constexpr (T == T_Q4_K || T == T_Q6_K) {
    if (pro == PRO_VEC && epi == EPI_XSUM) return launch_ring_t<T, PRO_VEC, EPI_XSUM>(p, s);
  }
  return cudaErrorInvalidValue;
}

static cudaError_t launch_ring(int type, int pro, int epi, const GemvParams& p, cudaStream_t s) {
  switch (type) {
    case T_TQ1_0: return launch_ring_pe<T_TQ1_0>(pro, epi, p, s);
    case T_TQ2_0: return launch_ring_pe<T_TQ2_0>(pro, epi, p, s);
    case T_Q4_K: return launch_ring_pe<T_Q4_K>(pro, epi, p, s);
    case T_Q6_K: return launch_ring_pe<T_Q6_K>(pro, epi, p, s);
    case T_Q8_0: return launch_ring_pe<T_Q8_0>(pro, epi, p, s);
    default: return cudaErrorInvalidValue;
  }
}


// ---------------------------------------------------------------------------
// resident-slice GEMV launch (layer matrices of ternary types)

// Smallest even unit with 16-byte aligned planes: the finest row granularity
// the packed layout allows, so the per-CTA runs come out even.
static int slice_unit_rows(int nb) {
  for (int U = 2; U <= 32; U += 2)
    if ((U * nb) % 8 == 0) return U;
  return -1;
}

template <int T, int PRO, int EPI>
static cudaError_t launch_slice_t(const GemvParams& p, const SliceGeom& g, int grid, cudaStream_t s) {
  auto kern = slice_kernel<T, PRO, EPI>;
  static size_t marks[kMaxDevices] = {};  // per instantiation
  cudaError_t e = opt_in_smem(kern, (size_t)SLICE_MAX_SMEM, marks);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(SLICE_THREADS);
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p, g);
}

template <int T>
static cudaError_t launch_slice_pe(int pro, int epi, const GemvParams& p, const SliceGeom& g, int grid,
                                   cudaStream_t s) {
  if (pro == PRO_VEC && epi == EPI_ADD) return launch_slice_t<T, PRO_VEC, EPI_ADD>(p, g, grid, s);
  if (pro == PRO_VEC && epi == EPI_STORE) return launch_slice_t<T, PRO_VEC, EPI_STORE>(p, g, grid, s);
  if (pro == PRO_NORM && epi == EPI_QKV) return launch_slice_t<T, PRO_NORM, EPI_QKV>(p, g, grid, s);
  if (pro == PRO_NORM && epi == EPI_SWIGLU) return launch_slice_t<T, PRO_NORM, EPI_SWIGLU>(p, g, grid, s);
  // tensor-parallel shards: the residual completed from the sums exchange,
  // and the row-parallel producers of both exchanges (p2p.cuh)
  if (pro == PRO_NFOLD && epi == EPI_QKV) return launch_slice_t<T, PRO_NFOLD, EPI_QKV>(p, g, grid, s);
  if (pro == PRO_NFOLD && epi == EPI_SWIGLU) return launch_slice_t<T, PRO_NFOLD, EPI_SWIGLU>(p, g, grid, s);
  if (pro == PRO_XAMAX && epi == EPI_XSUM) return launch_slice_t<T, PRO_XAMAX, EPI_XSUM>(p, g, grid, s);
  if (pro == PRO_XAMAX && epi == EPI_TERMS) return launch_slice_t<T, PRO_XAMAX, EPI_TERMS>(p, g, grid, s);
  if (pro == PRO_GSCALE && epi == EPI_TERMS) return launch_slice_t<T, PRO_GSCALE, EPI_TERMS>(p, g, grid, s);
  return cudaErrorInvalidValue;
}

static cudaError_t launch_slice(int type, int pro, int epi, const GemvParams& p, const SliceGeom& g,
                                int grid, cudaStream_t s) {
  switch (type) {
    case T_TQ1_0: return launch_slice_pe<T_TQ1_0>(pro, epi, p, g, grid, s);
    case T_TQ2_0: return launch_slice_pe<T_TQ2_0>(pro, epi, p, g, grid, s);
    default: return cudaErrorInvalidValue;
  }
}

template <int T, int PRO, int EPI>
static cudaError_t launch_stream_t(const GemvParams& p, const StreamGeom& g, int grid, cudaStream_t s) {
  auto kern = stream_kernel<T, PRO, EPI>;
  static size_t marks[kMaxDevices] = {};  // per instantiation
  cudaError_t e = opt_in_smem(kern, (size_t)STREAM_MAX_SMEM, marks);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(STREAM_THREADS);
  cfg.dynamicSmemBytes = g.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p, g);
}

template <int T>
static cudaError_t launch_stream_pe(int pro, int epi, const GemvParams& p, const StreamGeom& g, int grid,
                                    cudaStream_t s) {
  if (pro == PRO_VEC && epi == EPI_ADD) return launch_stream_t<T, PRO_VEC, EPI_ADD>(p, g, grid, s);
  if (pro == PRO_VEC && epi == EPI_STORE) return launch_stream_t<T, PRO_VEC, EPI_STORE>(p, g, grid, s);
  if (pro == PRO_NORM && epi == EPI_QKV) return launch_stream_t<T, PRO_NORM, EPI_QKV>(p, g, grid, s);
  if (pro == PRO_NORM && epi == EPI_SWIGLU) return launch_stream_t<T, PRO_NORM, EPI_SWIGLU>(p, g, grid, s);
  if (pro == PRO_NFOLD && epi == EPI_QKV) return launch_stream_t<T, PRO_NFOLD, EPI_QKV>(p, g, grid, s);
  if (pro == PRO_NFOLD && epi == EPI_SWIGLU) return launch_stream_t<T, PRO_NFOLD, EPI_SWIGLU>(p, g, grid, s);
  if (pro == PRO_XAMAX && epi == EPI_XSUM) return launch_stream_t<T, PRO_XAMAX, EPI_XSUM>(p, g, grid, s);
  if (pro == PRO_XAMAX && epi == EPI_TERMS) return launch_stream_t<T, PRO_XAMAX, EPI_TERMS>(p, g, grid, s);
  if (pro == PRO_GSCALE && epi == EPI_TERMS) return launch_stream_t<T, PRO_GSCALE, EPI_TERMS>(p, g, grid, s);
  return cudaErrorInvalidValue;
}


// ---------------------------------------------------------------------------
// kernel-level entry points

__global__ void quantize_vec_kernel(const float* __restrict__ x, int n, int8_t* __restrict__ q,
                                    float* __restrict__ scale) {
  __shared__ float red[32];
  float am = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) am = absmax_acc(am, x[i]);
  const float amax = block_reduce<float>(am, red, OpMax(), 0.0f);
  const bool nz = amax > 0.0f;
  const float inv = nz ? __fdiv_rn(127.0f, amax) : 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) q[i] = (int8_t)quant1(x[i], inv);
  if (threadIdx.x == 0) *scale = nz ? __fdiv_rn(amax, 127.0f) : 0.0f;
}

__global__ void expf_range_kernel(uint32_t first_bits, size_t n, float* __restrict__ out) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = expf_up(__uint_as_float(first_bits + (uint32_t)i));
}

extern "C" foxcuda_status foxcuda_expf_range(uint32_t first_bits, size_t n, float* out, void* stream) {
  if (!out || n == 0) return fail(FOXCUDA_ERR_ARG, "expf_range: null or empty");
  if (n - 1 > (size_t)(0xffffffffu - first_bits)) return fail(FOXCUDA_ERR_ARG, "expf_range: past the last bit pattern");
  const unsigned grid = (unsigned)std::min<size_t>((n + 255) / 256, (size_t)current_sms() * 16);
  expf_range_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(first_bits, n, out);
  CK(cudaGetLastError(), "expf_range launch");
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_quantize_activations_i8(const float* x, size_t n, int8_t* q,
                                                          float* scale, void* stream) {
  if (!x || !q || !scale || n == 0) return fail(FOXCUDA_ERR_ARG, "quantize: null or empty");
  if (n > (size_t)INT32_MAX) return fail(FOXCUDA_ERR_ARG, "quantize: vector too long");
  quantize_vec_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(x, (int)n, q, scale);
  CK(cudaGetLastError(), "quantize launch");
  return FOXCUDA_OK;
}

static foxcuda_status check_gemv_args(int type, const void* a, const void* w, size_t n_rows,
                                      size_t n_cols, const void* out, int* nb, int* U) {
  if (!a || !w || !out) return fail(FOXCUDA_ERR_ARG, "gemv: null pointer");
  if (n_rows == 0 || n_cols == 0) return fail(FOXCUDA_ERR_ARG, "gemv: empty matrix");
  if (!type_gemv_ok(type))
    return fail(FOXCUDA_ERR_UNSUPPORTED,
                "gemv: no kernel for ggml type %d; this build handles TQ1_0, TQ2_0, Q4_K, "
                "Q6_K and Q8_0", type);
  const int be = block_elems(type);
  if (n_cols % be)
    return fail(FOXCUDA_ERR_ARG, "gemv: %zu columns is not a multiple of the %d-element block",
                n_cols, be);
  if (type != T_Q8_0 && n_cols % 256)
    return fail(FOXCUDA_ERR_ARG, "gemv: %zu columns is not a multiple of 256", n_cols);
  if (n_rows > (size_t)INT32_MAX || n_cols > (1u << 20))
    return fail(FOXCUDA_ERR_ARG, "gemv: %zu x %zu is beyond this build's limits", n_rows, n_cols);
  *nb = (int)(n_cols / be);
  *U = unit_rows(type, *nb);
  if (*U < 0) return fail(FOXCUDA_ERR_UNSUPPORTED, "gemv: %zu columns has no unit layout", n_cols);
  return FOXCUDA_OK;
}

extern "C" size_t foxcuda_packed_bytes(int type, size_t n_rows, size_t n_cols) {
  if (!type_gemv_ok(type)) return 0;
  return n_rows * row_bytes(type, n_cols);
}

static cudaError_t pack_rows(int type, const void* src, size_t n_rows, int nb, int U, void* dst,
                             cudaStream_t s) {
  const long total = (long)n_rows * nb;
  const int grid = (int)std::min<long>((total + 255) / 256, 4096);
  pack_kernel<<<grid, 256, 0, s>>>(type, (const uint8_t*)src, (int)n_rows, nb, U, (uint8_t*)dst);
  return cudaGetLastError();
}

extern "C" foxcuda_status foxcuda_pack(int type, const void* src, size_t n_rows, size_t n_cols,
                                       void* packed, void* stream) {
  int nb, U;
  foxcuda_status st = check_gemv_args(type, src, src, n_rows, n_cols, packed, &nb, &U);
  if (st) return st;
  CK(pack_rows(type, src, n_rows, nb, U, packed, (cudaStream_t)stream), "pack launch");
  return FOXCUDA_OK;
}

static GemvParams gemv_base(int type, const void* packed, size_t n_rows, size_t n_cols, int nb, int U) {
  GemvParams p;
  memset(&p, 0, sizeof p);
  p.w = (const uint8_t*)packed;
  p.n_rows = (int)n_rows;
  p.K = (int)n_cols;
  p.nb = nb;
  p.U = U;
  return p;
}

extern "C" foxcuda_status foxcuda_gemv_packed(int type, const float* x, const void* packed,
                                              size_t n_rows, size_t n_cols, float* out,
                                              void* stream) {
  int nb, U;
  foxcuda_status st = check_gemv_args(type, x, packed, n_rows, n_cols, out, &nb, &U);
  if (st) return st;
  GemvParams p = gemv_base(type, packed, n_rows, n_cols, nb, U);
  p.x = x;
  p.out = out;
  CK(launch_ring(type, PRO_VEC, EPI_STORE, p, (cudaStream_t)stream), "gemv launch");
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_gemv(int type, const float* x, const void* w, size_t n_rows,
                                       size_t n_cols, float* out, void* stream) {
  int nb, U;
  foxcuda_status st = check_gemv_args(type, x, w, n_rows, n_cols, out, &nb, &U);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  void* scratch = nullptr;
  CK(cudaMallocAsync(&scratch, n_rows * row_bytes(type, n_cols), s), "gemv scratch");
  cudaError_t e = pack_rows(type, w, n_rows, nb, U, scratch, s);
  if (e == cudaSuccess) {
    GemvParams p = gemv_base(type, scratch, n_rows, n_cols, nb, U);
    p.x = x;
    p.out = out;
    e = launch_gemv(type, PRO_VEC, EPI_STORE, p, s);
  }
  cudaError_t e2 = cudaFreeAsync(scratch, s);
  if (e != cudaSuccess) return cuda_fail(e, "gemv");
  CK(e2, "gemv scratch free");
  return FOXCUDA_OK;
}

// foxcuda_gemv without any allocation: the repacked weights go to one
// file-scope device array instead of stream-ordered scratch. It is for callers
// that must not allocate:
// - a server that has reserved the device's memory for its own pool, so an
//   allocation here would either fail or take memory the pool counts on;
// - a decode loop that must not meet an out-of-memory error or an
//   allocator's latency halfway through a token;
// - a device or driver configuration without stream-ordered allocation.
// The array is part of the module image. The driver places it when the
// module loads, so the call itself never asks for memory.
//
// The first call on a device looks up the array's device address once, with
// that device current, and caches it. Make that first call before any stream
// capture. Nothing in the array has to start at zero or survive between
// calls: every byte the GEMV reads was written by the same call's pack
// launch. The array is shared, so calls whose work overlaps in time (two
// streams, or two host threads without ordering between them) overwrite each
// other's packed weights. Callers must order their calls, for instance on one
// stream.
static __device__ __align__(256) unsigned char g_noalloc_scratch[FOXCUDA_GEMV_NOALLOC_MAX_BYTES];
static std::mutex g_noalloc_mu;
static void* g_noalloc_addr[64];  // per device ordinal, filled by the first call

extern "C" foxcuda_status foxcuda_gemv_noalloc(int type, const float* x, const void* w,
                                               size_t n_rows, size_t n_cols, float* out,
                                               void* stream) {
  int nb, U;
  foxcuda_status st = check_gemv_args(type, x, w, n_rows, n_cols, out, &nb, &U);
  if (st) return st;
  const size_t need = n_rows * row_bytes(type, n_cols);
  if (need > (size_t)FOXCUDA_GEMV_NOALLOC_MAX_BYTES)
    return fail(FOXCUDA_ERR_ARG,
                "gemv_noalloc: the repacked %zu x %zu matrix needs %zu bytes; the static "
                "scratch holds %zu. Use foxcuda_gemv, or foxcuda_pack + foxcuda_gemv_packed",
                n_rows, n_cols, need, (size_t)FOXCUDA_GEMV_NOALLOC_MAX_BYTES);
  int dev = -1;
  CK(cudaGetDevice(&dev), "gemv_noalloc: current device");
  if (dev < 0 || dev >= (int)(sizeof g_noalloc_addr / sizeof g_noalloc_addr[0]))
    return fail(FOXCUDA_ERR_UNSUPPORTED, "gemv_noalloc: device ordinal %d is beyond 63", dev);
  void* scratch;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
      void* p = nullptr;
      CK(cudaGetSymbolAddress(&p, g_noalloc_scratch), "gemv_noalloc: scratch address");
      g_noalloc_addr[dev] = p;
    }
    scratch = g_noalloc_addr[dev];
  }
  cudaStream_t s = (cudaStream_t)stream;
  CK(pack_rows(type, w, n_rows, nb, U, scratch, s), "gemv_noalloc pack launch");
  GemvParams p = gemv_base(type, scratch, n_rows, n_cols, nb, U);
  p.x = x;
  p.out = out;
  CK(launch_gemv(type, PRO_VEC, EPI_STORE, p, s), "gemv_noalloc launch");
  return FOXCUDA_OK;
}

static foxcuda_status gemv_tq_i8(int type, const int8_t* q, const float* act_scale, const void* w,
                                 size_t n_rows, size_t n_cols, float* out, void* stream) {
  int nb, U;
  foxcuda_status st = check_gemv_args(type, q, w, n_rows, n_cols, out, &nb, &U);
  if (st) return st;
  if (!act_scale) return fail(FOXCUDA_ERR_ARG, "gemv: null activation scale");
  cudaStream_t s = (cudaStream_t)stream;
  void* scratch = nullptr;
  CK(cudaMallocAsync(&scratch, n_rows * row_bytes(type, n_cols), s), "gemv scratch");
  cudaError_t e = pack_rows(type, w, n_rows, nb, U, scratch, s);
  if (e == cudaSuccess) {
    GemvParams p = gemv_base(type, scratch, n_rows, n_cols, nb, U);
    p.xq = q;
    p.xq_scale = act_scale;
    p.out = out;
    e = launch_gemv(type, PRO_PREQ, EPI_STORE, p, s);
  }
  cudaError_t e2 = cudaFreeAsync(scratch, s);
  if (e != cudaSuccess) return cuda_fail(e, "gemv");
  CK(e2, "gemv scratch free");
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_gemv_tq1_i8(const int8_t* q, const float* act_scale,
                                              const void* w, size_t n_rows, size_t n_cols,
                                              float* out, void* stream) {
  return gemv_tq_i8(T_TQ1_0, q, act_scale, w, n_rows, n_cols, out, stream);
}
extern "C" foxcuda_status foxcuda_gemv_tq2_i8(const int8_t* q, const float* act_scale,
                                              const void* w, size_t n_rows, size_t n_cols,
                                              float* out, void* stream) {
  return gemv_tq_i8(T_TQ2_0, q, act_scale, w, n_rows, n_cols, out, stream);
}

// ---------------------------------------------------------------------------
// The error word of kernel-level calls: the tensor-core passes record a wait
// that gave up here (contexts have their own). foxcuda_kernel_errors reads
// and clears it. Its address is looked up once per device, by the first call
// that needs it.
static __device__ int g_kernel_err;
static std::mutex g_kernel_err_mu;
static int* g_kernel_err_addr[kMaxDevices];

static int* kernel_err_ptr() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_kernel_err_mu);
  if (!g_kernel_err_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_kernel_err) == cudaSuccess) g_kernel_err_addr[dev] = (int*)p;
  }
  return g_kernel_err_addr[dev];
}

extern "C" foxcuda_status foxcuda_kernel_errors(void* stream) {
  int* p = kernel_err_ptr();
  if (!p) return fail(FOXCUDA_ERR_INTERNAL, "kernel_errors: no device error word on the current device");
  CK(cudaStreamSynchronize((cudaStream_t)stream), "kernel_errors");
  int code = 0;
  CK(cudaMemcpy(&code, p, 4, cudaMemcpyDeviceToHost), "kernel_errors");
  if (!code) return FOXCUDA_OK;
  CK(cudaMemset(p, 0, 4), "kernel_errors");
  return fail(FOXCUDA_ERR_INTERNAL, "device: a bounded wait of a kernel-level tensor-core call gave up "
              "(code %d); that call's output is not valid", code);
}

// ---------------------------------------------------------------------------
// M-token ternary GEMM on the tensor cores (tc.cuh)

template <int NT, int D>
static cudaError_t launch_tc_td(const TcParams& p, cudaStream_t s) {
  const size_t smem = tc_smem_bytes(NT, p.nb);
  static size_t marks[kMaxDevices] = {};
  cudaError_t e = opt_in_smem(tc_tq2_kernel<NT, D>, smem, marks);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)((p.n_rows + TC_ROWS - 1) / TC_ROWS), (unsigned)((p.n_tok + NT - 1) / NT));
  tc_tq2_kernel<NT, D><<<grid, TC_THREADS, smem, s>>>(p);
  return cudaGetLastError();
}

// Two K blocks in flight per thread of the ternary tensor-core pass. Measured
// on one 4B layer against one and four: 172 / 188 / 172 us at 8 tokens,
// 226 / 313 / 236 at 64 (the prompt chunk), 494 / 476 / 518 at 512.
template <int NT>
static cudaError_t launch_tc_t(const TcParams& p, cudaStream_t s) {
  return launch_tc_td<NT, 2>(p, s);
}

// The token tile is the smallest MMA N that holds all tokens, up to 64.
static cudaError_t launch_tc(const TcParams& p, cudaStream_t s) {
  if (p.n_tok <= 8) return launch_tc_t<8>(p, s);
  if (p.n_tok <= 16) return launch_tc_t<16>(p, s);
  if (p.n_tok <= 32) return launch_tc_t<32>(p, s);
  return launch_tc_t<64>(p, s);
}

static foxcuda_status check_gemm_args(const int8_t* q, const float* act_scale, size_t n_tokens,
                                      const void* w, size_t n_rows, size_t n_cols, const float* out) {
  if (!q || !act_scale || !w || !out) return fail(FOXCUDA_ERR_ARG, "gemm: null pointer");
  if (n_tokens == 0 || n_rows == 0 || n_cols == 0) return fail(FOXCUDA_ERR_ARG, "gemm: empty input");
  if (n_cols % 256)
    return fail(FOXCUDA_ERR_ARG, "gemm: %zu columns is not a multiple of 256", n_cols);
  if (n_cols / 256 > (size_t)TC_MAX_NB || n_rows > (size_t)INT32_MAX || n_tokens > (1u << 20))
    return fail(FOXCUDA_ERR_ARG, "gemm: %zu tokens x %zu x %zu is beyond this build's limits",
                n_tokens, n_rows, n_cols);
  if ((uintptr_t)q % 16 || (uintptr_t)w % 16)
    return fail(FOXCUDA_ERR_ARG, "gemm: activations and weights must be 16-byte aligned");
  return FOXCUDA_OK;
}

static TcParams tc_params(const int8_t* q, const float* act_scale, size_t n_tokens, const void* packed,
                          size_t n_rows, size_t n_cols, int U, float* out) {
  TcParams p;
  p.w = (const uint8_t*)packed;
  p.xq = q;
  p.xs = act_scale;
  p.out = out;
  p.n_rows = (int)n_rows;
  p.K = (int)n_cols;
  p.nb = (int)(n_cols / 256);
  p.U = U;
  p.n_tok = (int)n_tokens;
  p.err = nullptr;
  return p;
}

extern "C" foxcuda_status foxcuda_gemm_tq2_i8_packed(const int8_t* q, const float* act_scale,
                                                     size_t n_tokens, const void* packed,
                                                     size_t n_rows, size_t n_cols, float* out,
                                                     void* stream) {
  foxcuda_status st = check_gemm_args(q, act_scale, n_tokens, packed, n_rows, n_cols, out);
  if (st) return st;
  const int U = unit_rows(T_TQ2_0, (int)(n_cols / 256));
  if (U < 0) return fail(FOXCUDA_ERR_UNSUPPORTED, "gemm: %zu columns has no unit layout", n_cols);
  TcParams p = tc_params(q, act_scale, n_tokens, packed, n_rows, n_cols, U, out);
  p.err = kernel_err_ptr();
  CK(launch_tc(p, (cudaStream_t)stream), "gemm launch");
  return FOXCUDA_OK;
}

template <int NT>
static cudaError_t launch_tc_split_t(const TcSplitParams& sp, cudaStream_t s) {
  const TcParams& p = sp.p;
  const size_t smem = tc_smem_bytes(NT, sp.bc);
  static size_t marks[kMaxDevices] = {};
  cudaError_t e = opt_in_smem(tc_tq2_split_kernel<NT>, smem, marks);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)((p.n_rows + TC_ROWS - 1) / TC_ROWS), (unsigned)((p.n_tok + NT - 1) / NT),
                  (unsigned)((p.nb + sp.bc - 1) / sp.bc));
  tc_tq2_split_kernel<NT><<<grid, TC_THREADS, smem, s>>>(sp);
  if ((e = cudaGetLastError())) return e;
  const size_t total = (size_t)p.n_tok * p.n_rows;
  tc_fold_kernel<<<(unsigned)std::min<size_t>((total + 255) / 256, 4096), 256, 0, s>>>(
      sp.terms, p.xs, p.n_rows, p.nb, p.n_tok, p.out);
  return cudaGetLastError();
}

// The blocks of a row are split so that the grid holds about two CTAs per SM.
static cudaError_t launch_tc_split(const TcParams& p, float* terms, cudaStream_t s) {
  const int nt = p.n_tok <= 8 ? 8 : p.n_tok <= 16 ? 16 : p.n_tok <= 32 ? 32 : 64;
  const int tiles = ((p.n_rows + TC_ROWS - 1) / TC_ROWS) * ((p.n_tok + nt - 1) / nt);
  const int splits = std::max(1, std::min(p.nb, (2 * current_sms() + tiles - 1) / tiles));
  TcSplitParams sp;
  sp.p = p;
  sp.terms = terms;
  sp.bc = (p.nb + splits - 1) / splits;
  if (nt == 8) return launch_tc_split_t<8>(sp, s);
  if (nt == 16) return launch_tc_split_t<16>(sp, s);
  if (nt == 32) return launch_tc_split_t<32>(sp, s);
  return launch_tc_split_t<64>(sp, s);
}

extern "C" foxcuda_status foxcuda_gemm_tq2_i8_split(const int8_t* q, const float* act_scale, size_t n_tokens,
                                                    const void* packed, size_t n_rows, size_t n_cols,
                                                    float* terms, float* out, void* stream) {
  foxcuda_status st = check_gemm_args(q, act_scale, n_tokens, packed, n_rows, n_cols, out);
  if (st) return st;
  if (!terms) return fail(FOXCUDA_ERR_ARG, "gemm: null terms scratch");
  const int U = unit_rows(T_TQ2_0, (int)(n_cols / 256));
  if (U < 0) return fail(FOXCUDA_ERR_UNSUPPORTED, "gemm: %zu columns has no unit layout", n_cols);
  TcParams p = tc_params(q, act_scale, n_tokens, packed, n_rows, n_cols, U, out);
  p.err = kernel_err_ptr();
  CK(launch_tc_split(p, terms, (cudaStream_t)stream), "gemm launch");
  return FOXCUDA_OK;
}

template <int T, int NT, int D>
static cudaError_t launch_kq_td(const TcKParams& p, cudaStream_t s) {
  const size_t smem = 2 * (size_t)tck_buf_bytes<T>(NT);
  static size_t marks[kMaxDevices] = {};
  cudaError_t e = opt_in_smem(tc_kq_kernel<T, NT, D>, smem, marks);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)((p.n_rows + TC_ROWS - 1) / TC_ROWS), (unsigned)((p.n_tok + NT - 1) / NT));
  tc_kq_kernel<T, NT, D><<<grid, TC_THREADS, smem, s>>>(p);
  return cudaGetLastError();
}

// one K block of look-ahead (the depth that was measured for this pass)
template <int T, int NT>
static cudaError_t launch_kq_t(const TcKParams& p, cudaStream_t s) {
  return launch_kq_td<T, NT, 1>(p, s);
}

// Token tiles: Q4_K up to 16 tokens (8 accumulators per block), Q6_K 8 (16).
static cudaError_t launch_kq(int type, const TcKParams& p, cudaStream_t s) {
  if (type == T_Q4_K) return p.n_tok <= 8 ? launch_kq_t<T_Q4_K, 8>(p, s) : launch_kq_t<T_Q4_K, 16>(p, s);
  if (type == T_Q6_K) return launch_kq_t<T_Q6_K, 8>(p, s);
  return cudaErrorInvalidValue;
}

extern "C" foxcuda_status foxcuda_gemm_kq_i8_packed(int type, const int8_t* q, const float* act_scales,
                                                    size_t n_tokens, const void* packed, size_t n_rows,
                                                    size_t n_cols, float* out, void* stream) {
  if (type != T_Q4_K && type != T_Q6_K)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "gemm: ggml type %d; the K-quant tensor-core pass takes Q4_K and Q6_K",
                type);
  foxcuda_status st = check_gemm_args(q, act_scales, n_tokens, packed, n_rows, n_cols, out);
  if (st) return st;
  const int nb = (int)(n_cols / 256);
  const int U = unit_rows(type, nb);
  if (U < 0) return fail(FOXCUDA_ERR_UNSUPPORTED, "gemm: %zu columns has no unit layout", n_cols);
  TcKParams p;
  p.w = (const uint8_t*)packed; p.xq = q; p.xs = act_scales; p.out = out; p.out_stride = (int)n_rows;
  p.n_rows = (int)n_rows; p.K = (int)n_cols; p.nb = nb; p.U = U; p.n_tok = (int)n_tokens; p.err = kernel_err_ptr();
  CK(launch_kq(type, p, (cudaStream_t)stream), "gemm launch");
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_gemm_kq_i8(int type, const int8_t* q, const float* act_scales,
                                             size_t n_tokens, const void* w, size_t n_rows, size_t n_cols,
                                             float* out, void* stream) {
  if (type != T_Q4_K && type != T_Q6_K)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "gemm: ggml type %d; the K-quant tensor-core pass takes Q4_K and Q6_K",
                type);
  foxcuda_status st = check_gemm_args(q, act_scales, n_tokens, w, n_rows, n_cols, out);
  if (st) return st;
  const int nb = (int)(n_cols / 256);
  const int U = unit_rows(type, nb);
  if (U < 0) return fail(FOXCUDA_ERR_UNSUPPORTED, "gemm: %zu columns has no unit layout", n_cols);
  cudaStream_t s = (cudaStream_t)stream;
  void* scratch = nullptr;
  CK(cudaMallocAsync(&scratch, n_rows * row_bytes(type, n_cols), s), "gemm scratch");
  cudaError_t e = pack_rows(type, w, n_rows, nb, U, scratch, s);
  if (e == cudaSuccess) {
    TcKParams p;
    p.w = (const uint8_t*)scratch; p.xq = q; p.xs = act_scales; p.out = out; p.out_stride = (int)n_rows;
    p.n_rows = (int)n_rows; p.K = (int)n_cols; p.nb = nb; p.U = U; p.n_tok = (int)n_tokens; p.err = kernel_err_ptr();
    e = launch_kq(type, p, s);
  }
  cudaError_t e2 = cudaFreeAsync(scratch, s);
  if (e != cudaSuccess) return cuda_fail(e, "gemm");
  CK(e2, "gemm scratch free");
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_gemm_tq_i8(int type, const int8_t* q, const float* act_scale,
                                             size_t n_tokens, const void* w, size_t n_rows,
                                             size_t n_cols, float* out, void* stream) {
  if (type != T_TQ1_0 && type != T_TQ2_0)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "gemm: ggml type %d; the tensor-core pass takes TQ1_0 and TQ2_0",
                type);
  foxcuda_status st = check_gemm_args(q, act_scale, n_tokens, w, n_rows, n_cols, out);
  if (st) return st;
  const int nb = (int)(n_cols / 256);
  const int U = unit_rows(T_TQ2_0, nb);
  if (U < 0) return fail(FOXCUDA_ERR_UNSUPPORTED, "gemm: %zu columns has no unit layout", n_cols);
  cudaStream_t s = (cudaStream_t)stream;
  const size_t tq2_bytes = n_rows * (size_t)nb * 66;
  const size_t tq1_bytes = type == T_TQ1_0 ? tq2_bytes : 0;  // the transcoded GGUF rows
  uint8_t* scratch = nullptr;
  CK(cudaMallocAsync((void**)&scratch, tq2_bytes + tq1_bytes, s), "gemm scratch");
  const void* rows = w;
  cudaError_t e = cudaSuccess;
  if (type == T_TQ1_0) {
    const long nblk = (long)n_rows * nb;
    tq1_to_tq2_kernel<<<(unsigned)((nblk + 127) / 128), 128, 0, s>>>((const uint8_t*)w, scratch + tq2_bytes,
                                                                     nblk);
    e = cudaGetLastError();
    rows = scratch + tq2_bytes;
  }
  if (e == cudaSuccess) e = pack_rows(T_TQ2_0, rows, n_rows, nb, U, scratch, s);
  if (e == cudaSuccess) {
    TcParams p = tc_params(q, act_scale, n_tokens, scratch, n_rows, n_cols, U, out);
    p.err = kernel_err_ptr();
    e = launch_tc(p, s);
  }
  cudaError_t e2 = cudaFreeAsync(scratch, s);
  if (e != cudaSuccess) return cuda_fail(e, "gemm");
  CK(e2, "gemm scratch free");
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_dequant_row(int type, const void* row, size_t n, float* out,
                                              void* stream) {
  if (!row || !out || n == 0) return fail(FOXCUDA_ERR_ARG, "dequant: null or empty");
  if (!(type == T_F32 || type == T_F16 || type == T_Q8_0 || type == T_Q4_K || type == T_Q6_K))
    return fail(FOXCUDA_ERR_UNSUPPORTED, "dequant: ggml type %d is not implemented", type);
  if (n % block_elems(type))
    return fail(FOXCUDA_ERR_ARG, "dequant: %zu elements is not a whole number of blocks", n);
  const int grid = (int)std::min<size_t>((n + 255) / 256, 1024);
  dequant_row_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(type, (const uint8_t*)row, (int)n, out);
  CK(cudaGetLastError(), "dequant launch");
  return FOXCUDA_OK;
}

static cudaError_t run_attention(const AttnParams& ap, bool exact, cudaStream_t s, bool pdl = false);

// Tile target of the tile attention (attn.cuh): about one tile per SM over
// all KV heads, at most one portable cluster (8) per KV head. Every path of
// a model (the decode step, prompt chunks, batches, tensor-parallel shards)
// uses the whole model's value, so they all cut the positions into the same
// tiles.
static int attn_nt_for(int sms, int n_kv_full) {
  return std::max(1, std::min(ATTN_TILE_MAX, sms / std::max(1, n_kv_full)));
}
// The tile attention's ring: rows per slot, the most (128, 64, 32 or 16)
// for which three slots and the score rows fit a CTA's shared memory
// (dynamic, below the 227 KB limit with room for the static arrays); and
// four slots instead of three when the CTA holds an SM alone anyway (more
// than half of it) and the fourth fits.
constexpr size_t ATTN_SMEM_MAX = 220 * 1024;
constexpr size_t ATTN_SMEM_PAIR = 110 * 1024;  // two CTAs per SM below this
static void attn_ring(AttnParams& ap, int gqa) {
  int ch = 128;
  while (ch > 16 && attn_tile_smem_bytes(ap.n_ctx, ap.nt, gqa, ap.hd, ap.kv_f16, ch, ATTN_RING_MIN) > ATTN_SMEM_MAX)
    ch >>= 1;
  ap.stage_rows = ch;
  ap.stage_slots = ATTN_RING_MIN;
  if (attn_tile_smem_bytes(ap.n_ctx, ap.nt, gqa, ap.hd, ap.kv_f16, ch, ATTN_RING_MIN) > ATTN_SMEM_PAIR &&
      attn_tile_smem_bytes(ap.n_ctx, ap.nt, gqa, ap.hd, ap.kv_f16, ch, ATTN_RING_MAX) <= ATTN_SMEM_MAX)
    ap.stage_slots = ATTN_RING_MAX;
}

extern "C" int foxcuda_attn_tile_target(int device, uint32_t n_head_kv) {
  return attn_nt_for(sm_count(device), (int)n_head_kv);
}

extern "C" foxcuda_status foxcuda_attention(const float* q, const void* kcache, const void* vcache,
                                            int kv_type, uint32_t n_head, uint32_t n_head_kv,
                                            uint32_t head_dim, uint32_t n_ctx, uint32_t pos,
                                            int exact, float* out, void* stream) {
  if (!q || !kcache || !vcache || !out) return fail(FOXCUDA_ERR_ARG, "attention: null pointer");
  if (kv_type != FOXCUDA_KV_F16 && kv_type != FOXCUDA_KV_F32)
    return fail(FOXCUDA_ERR_ARG, "attention: kv_type %d", kv_type);
  if (!n_head || !n_head_kv || n_head % n_head_kv || n_head / n_head_kv > ATTN_MAX_GQA ||
      head_dim % 32 || head_dim > 32 * ATTN_MAX_DPL || head_dim == 0)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "attention: %u heads / %u kv heads / head_dim %u not covered",
                n_head, n_head_kv, head_dim);
  if (pos >= n_ctx) return fail(FOXCUDA_ERR_ARG, "attention: position %u outside %u", pos, n_ctx);
  if (exact && n_ctx > 16384) return fail(FOXCUDA_ERR_UNSUPPORTED, "attention: exact mode holds 16384 positions");
  cudaStream_t s = (cudaStream_t)stream;
  const int nt = attn_nt_for(current_sms(), (int)n_head_kv);
  void* scratch = nullptr;
  CK(cudaMallocAsync(&scratch, 256, s), "attention scratch");
  int* pos_dev = (int*)scratch;
  cudaError_t e = cudaMemsetAsync(scratch, 0, 256, s);
  const int p32 = (int)pos;
  if (e == cudaSuccess) e = cudaMemcpyAsync(pos_dev, &p32, 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // p32 lives on this stack
  if (e == cudaSuccess) {
    AttnParams ap{};
    ap.q = q; ap.kcache = kcache; ap.vcache = vcache; ap.kv_f16 = kv_type == FOXCUDA_KV_F16;
    ap.n_ctx = (int)n_ctx; ap.hd = (int)head_dim; ap.n_head = (int)n_head; ap.n_kv = (int)n_head_kv;
    ap.nt = nt; ap.pos = pos_dev; ap.out = out;
    ap.scale = 1.0f / sqrtf((float)head_dim);
    e = run_attention(ap, exact != 0, s);
  }
  cudaError_t e2 = cudaFreeAsync(scratch, s);
  if (e != cudaSuccess) return cuda_fail(e, "attention");
  CK(e2, "attention scratch free");
  return FOXCUDA_OK;
}

// Integer partials straight from GGUF-layout blocks, through the same block
// decoders the GEMV kernels use (the block bytes are regrouped in registers
// into the plane order the decoders read).
template <int T>
__global__ void partials_kernel(const int8_t* __restrict__ q, const uint8_t* __restrict__ w,
                                int n_rows, int nb, int32_t* __restrict__ out) {
  const long g = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (g >= (long)n_rows * nb) return;
  const int b = (int)(g % nb);
  typename W<T>::R r;
  unsigned char* rb = reinterpret_cast<unsigned char*>(&r);
  memset(rb, 0, sizeof r);
  const SegTable tab = seg_table(T);
  const uint8_t* blk = w + g * block_bytes(T);
  int off = 0;
  for (int p = 0; p < tab.n; ++p) {
    for (int i = 0; i < tab.s[p].size; ++i) rb[off + i] = blk[tab.s[p].src + i];
    off += tab.s[p].size;
  }
  uint32_t xw[64];
  const uint32_t* src = reinterpret_cast<const uint32_t*>(q + (long)b * 256);
  for (int i = 0; i < 64; ++i) xw[i] = src[i];
  int sx = 0;
  for (int i = 0; i < 64; ++i) sx = dp4a(0x01010101u, xw[i], sx);
  if constexpr (T == T_TQ1_0 || T == T_TQ2_0) {
    out[g] = W<T>::isum(r, xw, sx);
  } else if constexpr (T == T_Q4_K) {
    W<T>::ipart(r, xw, out + g * 16);
  } else if constexpr (T == T_Q6_K) {
    W<T>::ipart(r, xw, out + g * 4);
  }
}

extern "C" foxcuda_status foxcuda_block_partials(int type, const int8_t* q, const void* w,
                                                 size_t n_rows, size_t n_cols, int32_t* out,
                                                 void* stream) {
  if (!q || !w || !out || n_rows == 0 || n_cols == 0)
    return fail(FOXCUDA_ERR_ARG, "partials: null pointer or empty matrix");
  if (n_cols % 256) return fail(FOXCUDA_ERR_ARG, "partials: columns not a multiple of 256");
  const int nb = (int)(n_cols / 256);
  const long total = (long)n_rows * nb;
  const int grid = (int)((total + 127) / 128);
  cudaStream_t s = (cudaStream_t)stream;
  switch (type) {
    case T_TQ1_0: partials_kernel<T_TQ1_0><<<grid, 128, 0, s>>>(q, (const uint8_t*)w, (int)n_rows, nb, out); break;
    case T_TQ2_0: partials_kernel<T_TQ2_0><<<grid, 128, 0, s>>>(q, (const uint8_t*)w, (int)n_rows, nb, out); break;
    case T_Q4_K: partials_kernel<T_Q4_K><<<grid, 128, 0, s>>>(q, (const uint8_t*)w, (int)n_rows, nb, out); break;
    case T_Q6_K: partials_kernel<T_Q6_K><<<grid, 128, 0, s>>>(q, (const uint8_t*)w, (int)n_rows, nb, out); break;
    default: return fail(FOXCUDA_ERR_UNSUPPORTED, "partials: ggml type %d has none", type);
  }
  CK(cudaGetLastError(), "partials launch");
  return FOXCUDA_OK;
}

// ---------------------------------------------------------------------------
// HBM weight store

struct PackedMat {
  int type = -1;
  int src_type = -1;  // GGUF type of the uploaded tensor (bytes are counted in it)
  int n_rows = 0, K = 0, nb = 0, U = 0;
  uint8_t* dev = nullptr;
  // row-per-lane Q8_0 head layout (rows.cuh)
  bool rows32 = false;
  // resident-slice launch (ternary layer matrices whose per-CTA run fits on
  // chip), or the streaming slice launch (larger ones)
  bool slice = false;
  bool stream = false;
  int pro = PRO_VEC;
  int grid = 0;
  SliceGeom g;
  StreamGeom sg;
};

// A ternary layer matrix through the slice kernel its plan chose.
static cudaError_t launch_sliced(const PackedMat& W, int pro, int epi, const GemvParams& p, cudaStream_t s) {
  if (W.slice) return launch_slice(W.type, pro, epi, p, W.g, W.grid, s);
  switch (W.type) {
    case T_TQ1_0: return launch_stream_pe<T_TQ1_0>(pro, epi, p, W.sg, W.grid, s);
    case T_TQ2_0: return launch_stream_pe<T_TQ2_0>(pro, epi, p, W.sg, W.grid, s);
    default: return cudaErrorInvalidValue;
  }
}

struct RawTensor {
  int type = -1;
  int src_type = -1;  // the GGUF type when the device holds a transcoded copy
  uint64_t ne0 = 0, ne1 = 0;
  uint8_t* dev = nullptr;
  size_t bytes = 0;
};

struct LayerW {
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  PackedMat qkv[3];  // [q|k|v] split into runs of one type; count in n_qkv
  int qkv_base[3] = {0, 0, 0};
  int n_qkv = 0;
  PackedMat o, gateup, down;
};

struct foxcuda_model {
  foxcuda_model_info info;     // the whole model (what uploads are checked against)
  foxcuda_model_info loc;      // this tensor-parallel shard (== info when tp_size == 1)
  int tp_rank = 0, tp_size = 1;
  uint32_t q_row0 = 0, kv_row0 = 0;        // first q row / k,v row of this shard
  uint32_t o_block0 = 0, o_blocks = 0;     // attn_output column blocks of this shard
  uint32_t f_block0 = 0, f_blocks = 0;     // FFN blocks (256 wide) of this shard
  uint32_t f_blocks_all[8] = {0};          // FFN blocks of every shard, rank order
  uint32_t vocab0 = 0;                     // first head row of this shard
  int device = 0;
  int attn_nt = 1;             // tile target of the tile attention (every path of this model)
  bool finalized = false;
  std::vector<RawTensor> raw;  // [role * (n_layer+1) + layer] staging until finalize
  RawTensor embd;              // GGUF layout, row gather
  float* out_norm = nullptr;
  PackedMat output;
  std::vector<LayerW> layers;
  uint64_t device_bytes = 0;
  std::vector<void*> allocs;
  RawTensor& slot(int role, uint32_t layer) { return raw[(size_t)role * (info.n_layer + 1) + layer]; }
};

static cudaError_t dev_alloc(foxcuda_model* m, size_t bytes, void** p) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e == cudaSuccess) { m->allocs.push_back(*p); m->device_bytes += bytes; }
  return e;
}

extern "C" foxcuda_status foxcuda_model_create(const foxcuda_model_info* info, int device,
                                               foxcuda_model** out) {
  if (!info || !out) return fail(FOXCUDA_ERR_ARG, "model: null argument");
  *out = nullptr;
  const foxcuda_model_info& mi = *info;
  if (!mi.n_layer || !mi.n_embd || !mi.n_head || !mi.n_head_kv || !mi.n_ff || !mi.n_vocab ||
      !mi.head_dim)
    return fail(FOXCUDA_ERR_FORMAT, "model: architecture metadata is incomplete");
  if (mi.head_dim % 2) return fail(FOXCUDA_ERR_UNSUPPORTED, "model: odd head dimension %u", mi.head_dim);
  if (mi.n_head % mi.n_head_kv)
    return fail(FOXCUDA_ERR_FORMAT, "model: %u query heads do not divide into %u kv heads",
                mi.n_head, mi.n_head_kv);
  if (mi.n_head / mi.n_head_kv > ATTN_MAX_GQA || mi.head_dim > 32 * ATTN_MAX_DPL ||
      mi.head_dim % 32)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "model: head_dim %u / gqa %u not covered by the "
                "attention kernel (head_dim a multiple of 32 up to 256, gqa <= 8)",
                mi.head_dim, mi.n_head / mi.n_head_kv);
  if (mi.n_embd % 256 || mi.n_ff % 256 || (mi.n_head * mi.head_dim) % 256)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "model: widths must be multiples of 256");
  foxcuda_status st = foxcuda_init(device);
  if (st) return st;
  foxcuda_model* m = new foxcuda_model();
  m->info = mi;
  m->loc = mi;
  m->o_blocks = mi.n_head * mi.head_dim / 256;
  m->f_blocks = mi.n_ff / 256;
  m->f_blocks_all[0] = m->f_blocks;
  m->device = device;
  m->attn_nt = attn_nt_for(sm_count(device), (int)mi.n_head_kv);
  m->raw.resize((size_t)FOXCUDA_N_ROLES * (mi.n_layer + 1));
  m->layers.resize(mi.n_layer);
  *out = m;
  return FOXCUDA_OK;
}

// Tensor-parallel shard tp_rank of tp_size (upstream has no multi-GPU path;
// the split is Megatron-style): q/k/v by heads, gate/up by 256-wide FFN blocks
// and the head by vocab rows (column-parallel, no exchange); attn_output and
// ffn_down by the matching column blocks (row-parallel: their block terms are
// exchanged and folded in upstream's block order, see foxcuda_tp_terms).
extern "C" foxcuda_status foxcuda_model_create_tp(const foxcuda_model_info* info, int device,
                                                  int tp_rank, int tp_size, foxcuda_model** out) {
  if (!info || !out) return fail(FOXCUDA_ERR_ARG, "model: null argument");
  if (tp_size < 1 || tp_size > 8 || tp_rank < 0 || tp_rank >= tp_size)
    return fail(FOXCUDA_ERR_ARG, "model: tensor-parallel rank %d of %d (at most 8 shards)", tp_rank, tp_size);
  const foxcuda_model_info& mi = *info;
  if (tp_size > 1) {
    if (mi.n_head % tp_size || mi.n_head_kv % tp_size)
      return fail(FOXCUDA_ERR_UNSUPPORTED, "model: %u query / %u kv heads do not split over %d shards",
                  mi.n_head, mi.n_head_kv, tp_size);
    if ((mi.n_head / tp_size * mi.head_dim) % 256)
      return fail(FOXCUDA_ERR_UNSUPPORTED, "model: a shard's attention output is not whole 256-blocks");
    if (mi.n_ff / 256 < (uint32_t)tp_size || mi.n_vocab % 32)
      return fail(FOXCUDA_ERR_UNSUPPORTED, "model: FFN or vocabulary too small to split %d ways", tp_size);
  }
  foxcuda_status st = foxcuda_model_create(info, device, out);
  if (st || tp_size == 1) return st;
  foxcuda_model* m = *out;
  m->tp_rank = tp_rank;
  m->tp_size = tp_size;
  const uint32_t hl = mi.n_head / tp_size, kvl = mi.n_head_kv / tp_size;
  m->loc.n_head = hl;
  m->loc.n_head_kv = kvl;
  m->q_row0 = tp_rank * hl * mi.head_dim;
  m->kv_row0 = tp_rank * kvl * mi.head_dim;
  m->o_blocks = hl * mi.head_dim / 256;
  m->o_block0 = tp_rank * m->o_blocks;
  const uint32_t nbf = mi.n_ff / 256;
  for (int k = 0; k < tp_size; ++k) m->f_blocks_all[k] = (k + 1) * nbf / tp_size - k * nbf / tp_size;
  m->f_block0 = tp_rank * nbf / tp_size;
  m->f_blocks = m->f_blocks_all[tp_rank];
  m->loc.n_ff = m->f_blocks * 256;
  const uint32_t per = (mi.n_vocab / tp_size + 31) / 32 * 32;
  m->vocab0 = std::min(mi.n_vocab, tp_rank * per);
  m->loc.n_vocab = std::min(mi.n_vocab, m->vocab0 + per) - m->vocab0;
  if (m->loc.n_vocab == 0) {
    foxcuda_model_destroy(m);
    *out = nullptr;
    return fail(FOXCUDA_ERR_UNSUPPORTED, "model: vocabulary too small to split %d ways", tp_size);
  }
  return FOXCUDA_OK;
}

extern "C" void foxcuda_model_destroy(foxcuda_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  for (void* p : m->allocs) cudaFree(p);
  for (RawTensor& r : m->raw) if (r.dev) cudaFree(r.dev);
  delete m;
}

extern "C" uint64_t foxcuda_model_device_bytes(const foxcuda_model* m) { return m ? m->device_bytes : 0; }

static bool role_per_layer(int role) { return role >= FOXCUDA_ATTN_NORM && role < FOXCUDA_N_ROLES; }

extern "C" foxcuda_status foxcuda_model_upload(foxcuda_model* m, int role, uint32_t layer,
                                               int type, uint64_t ne0, uint64_t ne1,
                                               const void* host, size_t bytes) {
  if (!m || !host) return fail(FOXCUDA_ERR_ARG, "upload: null argument");
  if (m->finalized) return fail(FOXCUDA_ERR_ARG, "upload: model already finalized");
  if (role < 0 || role >= FOXCUDA_N_ROLES) return fail(FOXCUDA_ERR_ARG, "upload: bad role %d", role);
  if (role_per_layer(role) ? layer >= m->info.n_layer : layer != 0)
    return fail(FOXCUDA_ERR_ARG, "upload: bad layer %u for role %d", layer, role);
  if (ne1 == 0) ne1 = 1;
  const size_t want = row_bytes(type, ne0) * ne1;
  if (!(type == T_F32 || type == T_F16 || type_gemv_ok(type)) || row_bytes(type, ne0) == 0)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "upload: ggml type %d with %llu columns", type,
                (unsigned long long)ne0);
  if (bytes != want)
    return fail(FOXCUDA_ERR_FORMAT, "upload: %zu bytes, the shape wants %zu", bytes, want);
  cudaSetDevice(m->device);
  RawTensor& r = m->slot(role, layer);
  if (r.dev) cudaFree(r.dev);
  r = RawTensor();
  CK(cudaMalloc(&r.dev, bytes), "upload alloc");
  r.type = type; r.ne0 = ne0; r.ne1 = ne1; r.bytes = bytes;
  CK(cudaMemcpy(r.dev, host, bytes, cudaMemcpyHostToDevice), "upload copy");
  return FOXCUDA_OK;
}

// foxcuda_model_upload with the tensor's bytes generated on the device
// (synthgen.cuh) from (seed, sigma) instead of copied from the host.
extern "C" foxcuda_status foxcuda_model_upload_synthetic(foxcuda_model* m, int role, uint32_t layer, int type,
                                                         uint64_t ne0, uint64_t ne1, uint64_t seed,
                                                         float sigma) {
  if (!m) return fail(FOXCUDA_ERR_ARG, "upload_synthetic: null model");
  if (m->finalized) return fail(FOXCUDA_ERR_ARG, "upload_synthetic: model already finalized");
  if (role < 0 || role >= FOXCUDA_N_ROLES) return fail(FOXCUDA_ERR_ARG, "upload_synthetic: bad role %d", role);
  if (role_per_layer(role) ? layer >= m->info.n_layer : layer != 0)
    return fail(FOXCUDA_ERR_ARG, "upload_synthetic: bad layer %u for role %d", layer, role);
  if (type != T_TQ1_0 && type != T_TQ2_0 && type != T_Q8_0 && type != T_Q4_K && type != T_Q6_K)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "upload_synthetic: no generator for ggml type %d (TQ1_0, TQ2_0, Q8_0, "
                "Q4_K, Q6_K)", type);
  if (!(sigma > 0.0f)) return fail(FOXCUDA_ERR_ARG, "upload_synthetic: sigma %g", sigma);
  if (ne1 == 0) ne1 = 1;
  const size_t rb = row_bytes(type, ne0);
  if (rb == 0) return fail(FOXCUDA_ERR_ARG, "upload_synthetic: %llu columns of type %d", (unsigned long long)ne0, type);
  const size_t bytes = rb * ne1;
  cudaSetDevice(m->device);
  RawTensor& r = m->slot(role, layer);
  if (r.dev) cudaFree(r.dev);
  r = RawTensor();
  CK(cudaMalloc(&r.dev, bytes), "upload alloc");
  r.type = type; r.ne0 = ne0; r.ne1 = ne1; r.bytes = bytes;
  const long n_blocks = (long)(bytes / block_bytes(type));
  const unsigned grid = (unsigned)std::max<long>(1, std::min<long>((n_blocks + 255) / 256, 32 * sm_count(m->device)));
  synth_fill_kernel<<<grid, 256>>>(type, r.dev, n_blocks, block_bytes(type), seed, (double)sigma);
  CK(cudaGetLastError(), "synthetic fill");
  CK(cudaDeviceSynchronize(), "synthetic fill");
  return FOXCUDA_OK;
}

static foxcuda_status pack_into(foxcuda_model* m, int type, const void* src_dev, int n_rows, int K,
                                PackedMat* out, int U = 0) {
  const int nb = K / block_elems(type);
  if (U <= 0) U = unit_rows(type, nb);
  if (U < 0) return fail(FOXCUDA_ERR_UNSUPPORTED, "pack: %d columns has no unit layout", K);
  void* dst = nullptr;
  CK(dev_alloc(m, (size_t)n_rows * row_bytes(type, K), &dst), "weight alloc");
  CK(pack_rows(type, src_dev, n_rows, nb, U, dst, 0), "pack");
  out->type = type; out->n_rows = n_rows; out->K = K; out->nb = nb; out->U = U;
  out->dev = (uint8_t*)dst;
  return FOXCUDA_OK;
}

static foxcuda_status norm_vec(foxcuda_model* m, const RawTensor& r, float** out) {
  const uint32_t n = m->info.n_embd;
  if (r.ne0 != n || r.ne1 != 1) return fail(FOXCUDA_ERR_FORMAT, "model: norm weight is not %u wide", n);
  if (r.type != T_F32 && r.type != T_F16)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "model: norm weights must be F32 or F16");
  void* d = nullptr;
  CK(dev_alloc(m, n * 4, &d), "norm alloc");
  dequant_row_kernel<<<(n + 255) / 256, 256>>>(r.type, r.dev, (int)n, (float*)d);
  CK(cudaGetLastError(), "norm convert");
  *out = (float*)d;
  return FOXCUDA_OK;
}

static void free_raw(RawTensor& r) {
  if (r.dev) cudaFree(r.dev);
  r = RawTensor();
}

// This shard's part of an uploaded matrix (rows r0.. of n, or column blocks
// b0.. of nb per row), replacing the staged tensor.
static foxcuda_status keep_rows(RawTensor& r, uint64_t r0, uint64_t n) {
  const size_t rb = row_bytes(r.type, r.ne0);
  void* d = nullptr;
  CK(cudaMalloc(&d, n * rb), "shard alloc");
  const cudaError_t e = cudaMemcpy(d, r.dev + r0 * rb, n * rb, cudaMemcpyDeviceToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "shard rows");
  }
  cudaFree(r.dev);
  r.dev = (uint8_t*)d; r.ne1 = n; r.bytes = n * rb;
  return FOXCUDA_OK;
}

static foxcuda_status keep_col_blocks(RawTensor& r, uint64_t b0, uint64_t nb) {
  const size_t rb = row_bytes(r.type, r.ne0);
  const size_t bb = row_bytes(r.type, 256) * nb;  // bytes of nb 256-wide blocks
  const size_t off = row_bytes(r.type, 256) * b0;
  void* d = nullptr;
  CK(cudaMalloc(&d, r.ne1 * bb), "shard alloc");
  const cudaError_t e = cudaMemcpy2D(d, bb, r.dev + off, rb, bb, r.ne1, cudaMemcpyDeviceToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "shard columns");
  }
  cudaFree(r.dev);
  r.dev = (uint8_t*)d; r.ne0 = nb * 256; r.bytes = r.ne1 * bb;
  return FOXCUDA_OK;
}

// TQ1_0 layer matrices are held as TQ2_0 (tq1_to_tq2_kernel): the same trits
// and scales, 66 instead of 54 bytes per block, and a quarter of the decode
// work per weight. Measured on the 4B step: 661 tok/s held as TQ2_0, 510
// decoding the GGUF TQ1_0 bytes.
static foxcuda_status transcode_tq1(RawTensor& r) {
  if (r.type != T_TQ1_0 || r.ne1 <= 1) return FOXCUDA_OK;
  const long nblk = (long)(r.bytes / 54);
  void* d = nullptr;
  CK(cudaMalloc(&d, (size_t)nblk * 66), "transcode alloc");
  tq1_to_tq2_kernel<<<(unsigned)((nblk + 127) / 128), 128>>>(r.dev, (uint8_t*)d, nblk);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_fail(e, "transcode");
  }
  cudaFree(r.dev);
  r.dev = (uint8_t*)d;
  r.bytes = (size_t)nblk * 66;
  r.type = T_TQ2_0;
  r.src_type = T_TQ1_0;
  return FOXCUDA_OK;
}

// The slice kernels' plan for a ternary layer matrix over one CTA per SM:
// resident when every CTA's run of units fits in shared memory (returns 1),
// else streamed in chunks through a ring of buffers (returns 2); 0 when
// neither fits.
static int slice_plan(const foxcuda_model* m, int type, int n_rows, int K, int U, int pro, int* grid_out,
                      SliceGeom* g_out, StreamGeom* sg_out) {
  const int sms = sm_count(m->device);
  const int units = n_rows / U;
  const int per = (units + sms - 1) / sms;
  const int grid = (units + per - 1) / per;
  if (grid_out) *grid_out = grid;
  const SliceGeom g = slice_geom(type, pro, n_rows, K, U, grid);
  if (g.smem <= SLICE_MAX_SMEM) {
    if (g_out) *g_out = g;
    return 1;
  }
  const StreamGeom sg = stream_geom(type, pro, n_rows, K, U, grid);
  if (sg.nbuf == 0) return 0;
  if (sg_out) *sg_out = sg;
  return 2;
}

// The slice kernels take a ternary layer matrix when its rows split into
// the slice unit and a plan fits a CTA's shared memory; returns that unit,
// or 0 for the unit kernel's layout.
static int slice_unit_for(const foxcuda_model* m, int type, int n_rows, int K, int pro) {
  if (type != T_TQ1_0 && type != T_TQ2_0) return 0;
  const int nb = K / 256;
  const int U = slice_unit_rows(nb);
  if (U < 0 || n_rows % U || (SLICE_THREADS / 2) / nb < 1) return 0;
  return slice_plan(m, type, n_rows, K, U, pro, nullptr, nullptr, nullptr) ? U : 0;
}

static void set_slice(const foxcuda_model* m, PackedMat* W, int pro) {
  const int plan = slice_plan(m, W->type, W->n_rows, W->K, W->U, pro, &W->grid, &W->g, &W->sg);
  W->pro = pro;
  W->slice = plan == 1;
  W->stream = plan == 2;
}

extern "C" foxcuda_status foxcuda_model_finalize(foxcuda_model* m) {
  if (!m) return fail(FOXCUDA_ERR_ARG, "finalize: null model");
  if (m->finalized) return FOXCUDA_OK;
  cudaSetDevice(m->device);
  const foxcuda_model_info& mi = m->info;
  const int nq = mi.n_head * mi.head_dim, nkv = mi.n_head_kv * mi.head_dim;
  const int E = mi.n_embd, Fd = mi.n_ff;
  static const char* names[] = {"token_embd", "output_norm", "output", "attn_norm", "attn_q",
                                "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate",
                                "ffn_up", "ffn_down"};
  struct Want { int role; uint64_t ne0, ne1; };
  const Want per_layer[] = {{FOXCUDA_ATTN_NORM, (uint64_t)E, 1}, {FOXCUDA_ATTN_Q, (uint64_t)E, (uint64_t)nq},
                            {FOXCUDA_ATTN_K, (uint64_t)E, (uint64_t)nkv}, {FOXCUDA_ATTN_V, (uint64_t)E, (uint64_t)nkv},
                            {FOXCUDA_ATTN_OUT, (uint64_t)nq, (uint64_t)E}, {FOXCUDA_FFN_NORM, (uint64_t)E, 1},
                            {FOXCUDA_FFN_GATE, (uint64_t)E, (uint64_t)Fd}, {FOXCUDA_FFN_UP, (uint64_t)E, (uint64_t)Fd},
                            {FOXCUDA_FFN_DOWN, (uint64_t)Fd, (uint64_t)E}};
  for (uint32_t l = 0; l < mi.n_layer; ++l)
    for (const Want& w : per_layer) {
      const RawTensor& r = m->slot(w.role, l);
      if (!r.dev) return fail(FOXCUDA_ERR_NOTFOUND, "model: tensor 'blk.%u.%s.weight' is missing", l, names[w.role]);
      if (r.ne0 != w.ne0 || r.ne1 != w.ne1)
        return fail(FOXCUDA_ERR_FORMAT, "model: 'blk.%u.%s.weight' is %llux%llu, expected %llux%llu", l,
                    names[w.role], (unsigned long long)r.ne0, (unsigned long long)r.ne1,
                    (unsigned long long)w.ne0, (unsigned long long)w.ne1);
      if (w.ne1 > 1 && !type_gemv_ok(r.type))
        return fail(FOXCUDA_ERR_UNSUPPORTED, "model: 'blk.%u.%s.weight' has ggml type %d, which has no "
                    "kernel here", l, names[w.role], r.type);
    }
  RawTensor& emb = m->slot(FOXCUDA_TOKEN_EMBD, 0);
  if (!emb.dev) return fail(FOXCUDA_ERR_NOTFOUND, "model: tensor 'token_embd.weight' is missing");
  if (emb.ne0 != (uint64_t)E || emb.ne1 != mi.n_vocab)
    return fail(FOXCUDA_ERR_FORMAT, "model: token_embd is %llux%llu, expected %ux%u",
                (unsigned long long)emb.ne0, (unsigned long long)emb.ne1, E, mi.n_vocab);
  if (!(emb.type == T_F32 || emb.type == T_F16 || emb.type == T_Q8_0 || emb.type == T_Q4_K ||
        emb.type == T_Q6_K))
    return fail(FOXCUDA_ERR_UNSUPPORTED, "model: token_embd type %d cannot be dequantised "
                "(upstream src/kernels.c:886-940)", emb.type);
  if (!m->slot(FOXCUDA_OUTPUT_NORM, 0).dev)
    return fail(FOXCUDA_ERR_NOTFOUND, "model: tensor 'output_norm.weight' is missing");
  RawTensor& outw = m->slot(FOXCUDA_OUTPUT, 0);
  const RawTensor& head = outw.dev ? outw : emb;  // tied output (upstream src/model.c:248-252)
  if (head.ne0 != (uint64_t)E || head.ne1 != mi.n_vocab)
    return fail(FOXCUDA_ERR_FORMAT, "model: output head is not %ux%u", E, mi.n_vocab);
  if (!type_gemv_ok(head.type))
    return fail(FOXCUDA_ERR_UNSUPPORTED, "model: output head type %d has no kernel here", head.type);

  foxcuda_status st;
  // this shard's widths (the whole model when tp_size == 1)
  const bool tp = m->tp_size > 1;
  const int nq_l = m->loc.n_head * mi.head_dim, nkv_l = m->loc.n_head_kv * mi.head_dim;
  const int Fd_l = m->loc.n_ff;
  for (uint32_t l = 0; l < mi.n_layer; ++l) {
    LayerW& L = m->layers[l];
    if (tp) {
      if ((st = keep_rows(m->slot(FOXCUDA_ATTN_Q, l), m->q_row0, nq_l))) return st;
      if ((st = keep_rows(m->slot(FOXCUDA_ATTN_K, l), m->kv_row0, nkv_l))) return st;
      if ((st = keep_rows(m->slot(FOXCUDA_ATTN_V, l), m->kv_row0, nkv_l))) return st;
      if ((st = keep_col_blocks(m->slot(FOXCUDA_ATTN_OUT, l), m->o_block0, m->o_blocks))) return st;
      if ((st = keep_rows(m->slot(FOXCUDA_FFN_GATE, l), (uint64_t)m->f_block0 * 256, Fd_l))) return st;
      if ((st = keep_rows(m->slot(FOXCUDA_FFN_UP, l), (uint64_t)m->f_block0 * 256, Fd_l))) return st;
      if ((st = keep_col_blocks(m->slot(FOXCUDA_FFN_DOWN, l), m->f_block0, m->f_blocks))) return st;
    }
    for (int role : {FOXCUDA_ATTN_Q, FOXCUDA_ATTN_K, FOXCUDA_ATTN_V, FOXCUDA_ATTN_OUT,
                     FOXCUDA_FFN_GATE, FOXCUDA_FFN_UP, FOXCUDA_FFN_DOWN})
      if ((st = transcode_tq1(m->slot(role, l)))) return st;
    if ((st = norm_vec(m, m->slot(FOXCUDA_ATTN_NORM, l), &L.attn_norm))) return st;
    if ((st = norm_vec(m, m->slot(FOXCUDA_FFN_NORM, l), &L.ffn_norm))) return st;
    // q|k|v: rows concatenated; consecutive tensors of one type share a matrix
    const RawTensor* qkv[3] = {&m->slot(FOXCUDA_ATTN_Q, l), &m->slot(FOXCUDA_ATTN_K, l),
                               &m->slot(FOXCUDA_ATTN_V, l)};
    const int rows[3] = {nq_l, nkv_l, nkv_l};
    int i = 0, base = 0;
    L.n_qkv = 0;
    while (i < 3) {
      int j = i, nrow = 0;
      size_t bytes = 0;
      while (j < 3 && qkv[j]->type == qkv[i]->type) { nrow += rows[j]; bytes += qkv[j]->bytes; ++j; }
      void* cat = nullptr;
      CK(cudaMalloc(&cat, bytes), "staging alloc");
      size_t off = 0;
      cudaError_t e = cudaSuccess;
      for (int k = i; k < j && e == cudaSuccess; ++k) {
        e = cudaMemcpy((uint8_t*)cat + off, qkv[k]->dev, qkv[k]->bytes, cudaMemcpyDeviceToDevice);
        off += qkv[k]->bytes;
      }
      if (e != cudaSuccess) {
        cudaFree(cat);
        return cuda_fail(e, "q|k|v concatenation");
      }
      int su = slice_unit_for(m, qkv[i]->type, nrow, E, PRO_NORM);
      for (int k = i; k < j && su; ++k)
        if (rows[k] % su) su = 0;
      st = pack_into(m, qkv[i]->type, cat, nrow, E, &L.qkv[L.n_qkv], su);
      L.qkv[L.n_qkv].src_type = qkv[i]->src_type;
      if (!st && su) set_slice(m, &L.qkv[L.n_qkv], PRO_NORM);
      cudaDeviceSynchronize();
      cudaFree(cat);
      if (st) return st;
      if (L.qkv[L.n_qkv].U > 0 && ((rows[i] % L.qkv[L.n_qkv].U) || (mi.head_dim % 2)))
        return fail(FOXCUDA_ERR_UNSUPPORTED, "model: q/k/v rows do not align to %d-row units",
                    L.qkv[L.n_qkv].U);
      L.qkv_base[L.n_qkv] = base;
      base += nrow;
      L.n_qkv++;
      i = j;
    }
    {
      // row-parallel shards take the slice layout too: the slice kernel
      // emits their block terms or row sums (foxcuda_tp_terms,
      // foxcuda_tp_p2p_row)
      const RawTensor& o = m->slot(FOXCUDA_ATTN_OUT, l);
      const int su = slice_unit_for(m, o.type, E, nq_l, PRO_VEC);
      if ((st = pack_into(m, o.type, o.dev, E, nq_l, &L.o, su))) return st;
      L.o.src_type = o.src_type;
      if (su) set_slice(m, &L.o, PRO_VEC);
    }
    // gate|up interleaved per unit: U/2 gate rows then the same U/2 up rows
    const RawTensor& g = m->slot(FOXCUDA_FFN_GATE, l);
    const RawTensor& u = m->slot(FOXCUDA_FFN_UP, l);
    if (g.type != u.type)
      return fail(FOXCUDA_ERR_UNSUPPORTED, "model: ffn_gate and ffn_up types differ in layer %u", l);
    {
      const int nb = E / block_elems(g.type);
      const int su = slice_unit_for(m, g.type, 2 * Fd_l, E, PRO_NORM);
      const int U = su ? su : unit_rows(g.type, nb);
      if (U < 0 || Fd_l % (U / 2)) return fail(FOXCUDA_ERR_UNSUPPORTED, "model: ffn width %d vs unit %d", Fd_l, U);
      const size_t rb = row_bytes(g.type, E), half = (size_t)(U / 2) * rb;
      void* cat = nullptr;
      CK(cudaMalloc(&cat, g.bytes + u.bytes), "staging alloc");
      cudaError_t e = cudaMemcpy2D(cat, 2 * half, g.dev, half, half, Fd_l / (U / 2), cudaMemcpyDeviceToDevice);
      if (e == cudaSuccess)
        e = cudaMemcpy2D((uint8_t*)cat + half, 2 * half, u.dev, half, half, Fd_l / (U / 2),
                         cudaMemcpyDeviceToDevice);
      if (e != cudaSuccess) {
        cudaFree(cat);
        return cuda_fail(e, "interleave");
      }
      st = pack_into(m, g.type, cat, 2 * Fd_l, E, &L.gateup, U);
      L.gateup.src_type = g.src_type;
      if (!st && su) set_slice(m, &L.gateup, PRO_NORM);
      cudaDeviceSynchronize();
      cudaFree(cat);
      if (st) return st;
    }
    {
      const RawTensor& d = m->slot(FOXCUDA_FFN_DOWN, l);
      const int su = slice_unit_for(m, d.type, E, Fd_l, PRO_VEC);
      if ((st = pack_into(m, d.type, d.dev, E, Fd_l, &L.down, su))) return st;
      L.down.src_type = d.src_type;
      if (su) set_slice(m, &L.down, PRO_VEC);
    }
    CK(cudaDeviceSynchronize(), "finalize layer");
    for (int role = FOXCUDA_ATTN_NORM; role < FOXCUDA_N_ROLES; ++role) free_raw(m->slot(role, l));
  }
  if ((st = norm_vec(m, m->slot(FOXCUDA_OUTPUT_NORM, 0), &m->out_norm))) return st;
  // this shard's head rows (all of them when tp_size == 1)
  const uint32_t nv_l = m->loc.n_vocab;
  const uint8_t* head_rows = head.dev + (size_t)m->vocab0 * row_bytes(head.type, E);
  if (head.type == T_Q8_0 && nv_l % 32 == 0) {
    // the row-per-lane layout of q8_rows_kernel
    PackedMat& H = m->output;
    void* dst = nullptr;
    CK(dev_alloc(m, (size_t)nv_l * row_bytes(T_Q8_0, E), &dst), "head alloc");
    const long total = (long)nv_l * (E / 32);
    pack_q8_rows32_kernel<<<(unsigned)std::min<long>((total + 255) / 256, 8192), 256>>>(
        head_rows, (int)nv_l, E / 32, (uint8_t*)dst);
    CK(cudaGetLastError(), "head pack");
    H.type = T_Q8_0; H.n_rows = (int)nv_l; H.K = E; H.nb = E / 32; H.U = 32;
    H.dev = (uint8_t*)dst; H.rows32 = true;
  } else if ((st = pack_into(m, head.type, head_rows, nv_l, E, &m->output))) {
    return st;
  }
  CK(cudaDeviceSynchronize(), "finalize head");
  m->embd = emb;
  m->device_bytes += emb.bytes;
  m->allocs.push_back(emb.dev);  // freed with the model
  emb = RawTensor();  // ownership moves to m->embd
  free_raw(outw);
  free_raw(m->slot(FOXCUDA_OUTPUT_NORM, 0));
  m->finalized = true;
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_model_get_info(const foxcuda_model* m, foxcuda_model_info* out) {
  if (!m || !out) return fail(FOXCUDA_ERR_ARG, "model_get_info: null argument");
  *out = m->info;
  return FOXCUDA_OK;
}

// ---------------------------------------------------------------------------
// device images: a finalized model's HBM layout in one file
//
// Upstream's repacker (fox_repack_gguf, src/repack.c:170-315) rewrites a GGUF
// so that each layer's tensors form one contiguous span, which its loader
// then maps instead of gathering. The device image goes one step further: the
// file holds the bytes exactly as they sit in HBM after finalize (TQ1_0
// layers already held as TQ2_0, q|k|v concatenated, gate|up interleaved,
// every matrix in its packed unit layout, norms as floats). Opening one is a
// sequential read through two pinned buffers into one device allocation,
// with no packing kernel and no staging copy on the device.
//
// Layout (little-endian): ImgHeader, n_entries ImgEntry, zero padding up to
// data_off (a multiple of 4096), then the data section. Entry offsets are
// relative to data_off and multiples of 256.

namespace {

constexpr char kImgMagic[8] = {'F', 'O', 'X', 'D', 'I', 'M', 'G', '1'};
constexpr uint32_t kImgVersion = 1;
enum ImgKind : uint32_t {
  IK_EMBD = 0, IK_OUT_NORM, IK_OUTPUT, IK_ATTN_NORM, IK_FFN_NORM, IK_QKV, IK_O, IK_GATEUP, IK_DOWN, IK_N
};
constexpr uint32_t IMG_ROWS32 = 1, IMG_SLICE = 2;

struct ImgHeader {
  char magic[8];
  uint32_t version, n_entries;
  uint64_t data_off, data_bytes;
  uint32_t sm_count, tp_rank, tp_size, vocab0;
  foxcuda_model_info info, loc;
  uint32_t q_row0, kv_row0, o_block0, o_blocks, f_block0, f_blocks, f_blocks_all[8];
  uint64_t table_hash;  // FNV-1a 64 of the entry table
};
struct ImgEntry {
  uint32_t kind, layer, index, flags;
  int32_t type, src_type, n_rows, K, nb, U, pro, qkv_base;
  uint64_t ne0, ne1;  // the embedding's GGUF shape
  uint64_t offset, bytes;
};
static_assert(sizeof(ImgHeader) == 184 && sizeof(ImgEntry) == 80, "image records have no padding");
static_assert(FOXCUDA_KV_PAGE == KV_PAGE, "the header's page size is the kernels'");

constexpr size_t kImgChunk = 64ull << 20;  // bytes per pinned staging buffer

uint64_t fnv1a(const void* p, size_t n) {
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < n; ++i) h = (h ^ reinterpret_cast<const uint8_t*>(p)[i]) * 1099511628211ull;
  return h;
}

size_t mat_bytes(const PackedMat& W) { return (size_t)W.n_rows * row_bytes(W.type, W.K); }

ImgEntry mat_entry(const PackedMat& W) {
  ImgEntry e{};
  e.type = W.type; e.src_type = W.src_type; e.n_rows = W.n_rows; e.K = W.K; e.nb = W.nb; e.U = W.U;
  e.pro = W.pro;
  e.flags = (W.rows32 ? IMG_ROWS32 : 0u) | ((W.slice || W.stream) ? IMG_SLICE : 0u);
  return e;
}

// Pinned staging buffers, a copy stream and an event per buffer, released on
// every path (after the stream has drained).
struct Staging {
  void* buf[2] = {nullptr, nullptr};
  cudaStream_t s = nullptr;
  cudaEvent_t ev[2] = {nullptr, nullptr};
  ~Staging() {
    if (s) cudaStreamSynchronize(s);
    for (int i = 0; i < 2; ++i) {
      if (buf[i]) cudaFreeHost(buf[i]);
      if (ev[i]) cudaEventDestroy(ev[i]);
    }
    if (s) cudaStreamDestroy(s);
  }
  cudaError_t init(int n_buf) {
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    for (int i = 0; i < n_buf && e == cudaSuccess; ++i) {
      e = cudaMallocHost(&buf[i], kImgChunk);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
    }
    return e;
  }
};

struct FileCloser {
  void operator()(FILE* f) const {
    if (f) fclose(f);
  }
};

}  // namespace

extern "C" foxcuda_status foxcuda_model_save_image(const foxcuda_model* m, const char* path) {
  if (!m || !path) return fail(FOXCUDA_ERR_ARG, "save_image: null argument");
  if (!m->finalized) return fail(FOXCUDA_ERR_ARG, "save_image: finalize the model first");
  struct Src { ImgEntry e; const void* dev; };
  std::vector<Src> src;
  uint64_t off = 0;
  auto add = [&](uint32_t kind, uint32_t layer, uint32_t index, const void* dev, uint64_t bytes, ImgEntry e) {
    e.kind = kind; e.layer = layer; e.index = index; e.offset = off; e.bytes = bytes;
    off = (off + bytes + 255) / 256 * 256;
    src.push_back({e, dev});
  };
  const uint64_t E = m->info.n_embd;
  {
    ImgEntry e{};
    e.type = m->embd.type; e.src_type = m->embd.src_type; e.ne0 = m->embd.ne0; e.ne1 = m->embd.ne1;
    add(IK_EMBD, 0, 0, m->embd.dev, m->embd.bytes, e);
  }
  add(IK_OUT_NORM, 0, 0, m->out_norm, E * 4, ImgEntry{});
  add(IK_OUTPUT, 0, 0, m->output.dev, mat_bytes(m->output), mat_entry(m->output));
  for (uint32_t l = 0; l < m->info.n_layer; ++l) {
    const LayerW& L = m->layers[l];
    add(IK_ATTN_NORM, l, 0, L.attn_norm, E * 4, ImgEntry{});
    add(IK_FFN_NORM, l, 0, L.ffn_norm, E * 4, ImgEntry{});
    for (int i = 0; i < L.n_qkv; ++i) {
      ImgEntry e = mat_entry(L.qkv[i]);
      e.qkv_base = L.qkv_base[i];
      add(IK_QKV, l, (uint32_t)i, L.qkv[i].dev, mat_bytes(L.qkv[i]), e);
    }
    add(IK_O, l, 0, L.o.dev, mat_bytes(L.o), mat_entry(L.o));
    add(IK_GATEUP, l, 0, L.gateup.dev, mat_bytes(L.gateup), mat_entry(L.gateup));
    add(IK_DOWN, l, 0, L.down.dev, mat_bytes(L.down), mat_entry(L.down));
  }
  std::vector<ImgEntry> table;
  for (const Src& s : src) table.push_back(s.e);
  ImgHeader h;
  memset(&h, 0, sizeof h);
  memcpy(h.magic, kImgMagic, 8);
  h.version = kImgVersion;
  h.n_entries = (uint32_t)table.size();
  h.data_off = (sizeof h + table.size() * sizeof(ImgEntry) + 4095) / 4096 * 4096;
  h.data_bytes = off;
  h.sm_count = (uint32_t)sm_count(m->device);
  h.tp_rank = (uint32_t)m->tp_rank; h.tp_size = (uint32_t)m->tp_size; h.vocab0 = m->vocab0;
  h.info = m->info; h.loc = m->loc;
  h.q_row0 = m->q_row0; h.kv_row0 = m->kv_row0; h.o_block0 = m->o_block0; h.o_blocks = m->o_blocks;
  h.f_block0 = m->f_block0; h.f_blocks = m->f_blocks;
  memcpy(h.f_blocks_all, m->f_blocks_all, sizeof h.f_blocks_all);
  h.table_hash = fnv1a(table.data(), table.size() * sizeof(ImgEntry));

  std::unique_ptr<FILE, FileCloser> f(fopen(path, "wb"));
  if (!f) return fail(FOXCUDA_ERR_IO, "save_image: cannot create %s: %s", path, strerror(errno));
  static const uint8_t zeros[4096] = {0};
  auto put = [&](const void* p, size_t n) { return fwrite(p, 1, n, f.get()) == n; };
  auto pad = [&](uint64_t n) {
    while (n > 0) {
      const size_t k = (size_t)std::min<uint64_t>(n, sizeof zeros);
      if (!put(zeros, k)) return false;
      n -= k;
    }
    return true;
  };
  auto io_fail = [&]() { return fail(FOXCUDA_ERR_IO, "save_image: writing %s: %s", path, strerror(errno)); };
  const uint64_t head_bytes = sizeof h + table.size() * sizeof(ImgEntry);
  if (!put(&h, sizeof h) || !put(table.data(), table.size() * sizeof(ImgEntry)) || !pad(h.data_off - head_bytes))
    return io_fail();
  cudaSetDevice(m->device);
  Staging st;
  CK(st.init(1), "save_image staging");
  uint64_t pos = 0;
  for (const Src& s : src) {
    if (!pad(s.e.offset - pos)) return io_fail();
    for (uint64_t done = 0; done < s.e.bytes;) {
      const size_t n = (size_t)std::min<uint64_t>(kImgChunk, s.e.bytes - done);
      CK(cudaMemcpyAsync(st.buf[0], (const uint8_t*)s.dev + done, n, cudaMemcpyDeviceToHost, st.s),
         "save_image copy");
      CK(cudaStreamSynchronize(st.s), "save_image copy");
      if (!put(st.buf[0], n)) return io_fail();
      done += n;
    }
    pos = s.e.offset + s.e.bytes;
  }
  if (!pad(h.data_bytes - pos)) return io_fail();
  if (fclose(f.release()) != 0) return fail(FOXCUDA_ERR_IO, "save_image: closing %s: %s", path, strerror(errno));
  return FOXCUDA_OK;
}

// Every check of an image that needs no device: the table against its hash,
// each entry's place in the data, and its shape against the model (shard)
// the header describes.
static foxcuda_status check_image(const ImgHeader& h, const std::vector<ImgEntry>& t, const char* path) {
  const foxcuda_model_info& mi = h.info;
  const foxcuda_model_info& lo = h.loc;
  if (h.tp_size < 1 || h.tp_size > 8 || h.tp_rank >= h.tp_size)
    return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: shard %u of %u", path, h.tp_rank, h.tp_size);
  if (fnv1a(t.data(), t.size() * sizeof(ImgEntry)) != h.table_hash)
    return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: the tensor table is corrupt", path);
  const uint64_t E = mi.n_embd;
  const int nq = (int)(lo.n_head * mi.head_dim), nkv = (int)(lo.n_head_kv * mi.head_dim);
  std::vector<int> seen((size_t)IK_N * (mi.n_layer + 1), 0);
  std::vector<int> qkv_runs(mi.n_layer, 0), qkv_rows(mi.n_layer, 0);
  for (size_t i = 0; i < t.size(); ++i) {
    const ImgEntry& e = t[i];
    const bool per_layer = e.kind == IK_ATTN_NORM || e.kind == IK_FFN_NORM || e.kind == IK_QKV ||
                           e.kind == IK_O || e.kind == IK_GATEUP || e.kind == IK_DOWN;
    if (e.kind >= IK_N || (per_layer ? e.layer >= mi.n_layer : e.layer != 0))
      return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: entry %zu has kind %u, layer %u", path, i, e.kind, e.layer);
    if (e.offset % 256 || e.offset > h.data_bytes || e.bytes > h.data_bytes - e.offset)
      return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: entry %zu lies outside the data", path, i);
    if (e.kind == IK_QKV) {
      if (e.index >= 3 || e.index != (uint32_t)qkv_runs[e.layer] || e.qkv_base != qkv_rows[e.layer])
        return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: q|k|v run %u of layer %u is out of order", path,
                    e.index, e.layer);
      qkv_runs[e.layer]++;
      qkv_rows[e.layer] += e.n_rows;
    } else if (e.index != 0 || seen[(size_t)e.kind * (mi.n_layer + 1) + e.layer]++) {
      return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: entry %zu repeats kind %u of layer %u", path, i, e.kind,
                  e.layer);
    }
    if (e.kind == IK_OUT_NORM || e.kind == IK_ATTN_NORM || e.kind == IK_FFN_NORM) {
      if (e.bytes != E * 4)
        return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: a norm is not %llu floats", path, (unsigned long long)E);
    } else if (e.kind == IK_EMBD) {
      if (e.ne0 != E || e.ne1 != mi.n_vocab || row_bytes(e.type, e.ne0) == 0 ||
          e.bytes != e.ne1 * row_bytes(e.type, e.ne0))
        return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: the embedding is not %llux%u", path,
                    (unsigned long long)E, mi.n_vocab);
    } else {
      if (!type_gemv_ok(e.type) || e.n_rows <= 0 || e.K <= 0 || e.U <= 0 || row_bytes(e.type, e.K) == 0 ||
          e.nb != e.K / block_elems(e.type) || e.bytes != (uint64_t)e.n_rows * row_bytes(e.type, e.K))
        return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: matrix entry %zu (type %d, %d x %d) is inconsistent",
                    path, i, e.type, e.n_rows, e.K);
      bool ok = true;
      if (e.kind == IK_OUTPUT) ok = e.K == (int)E && e.n_rows == (int)lo.n_vocab;
      if (e.kind == IK_QKV) ok = e.K == (int)E && qkv_rows[e.layer] <= nq + 2 * nkv;
      if (e.kind == IK_O) ok = e.K == nq && e.n_rows == (int)E;
      if (e.kind == IK_GATEUP) ok = e.K == (int)E && e.n_rows == 2 * (int)lo.n_ff;
      if (e.kind == IK_DOWN) ok = e.K == (int)lo.n_ff && e.n_rows == (int)E;
      if (!ok)
        return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: matrix entry %zu (%d x %d) does not fit the model",
                    path, i, e.n_rows, e.K);
    }
  }
  for (uint32_t k : {IK_EMBD, IK_OUT_NORM, IK_OUTPUT})
    if (!seen[(size_t)k * (mi.n_layer + 1)])
      return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: entry kind %u is missing", path, k);
  for (uint32_t l = 0; l < mi.n_layer; ++l) {
    for (uint32_t k : {IK_ATTN_NORM, IK_FFN_NORM, IK_O, IK_GATEUP, IK_DOWN})
      if (!seen[(size_t)k * (mi.n_layer + 1) + l])
        return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: layer %u lacks entry kind %u", path, l, k);
    if (qkv_rows[l] != nq + 2 * nkv)
      return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: layer %u has %d q|k|v rows, not %d", path, l,
                  qkv_rows[l], nq + 2 * nkv);
  }
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_model_open_image(const char* path, int device, foxcuda_model** out) {
  if (!path || !out) return fail(FOXCUDA_ERR_ARG, "open_image: null argument");
  *out = nullptr;
  std::unique_ptr<FILE, FileCloser> f(fopen(path, "rb"));
  if (!f) return fail(FOXCUDA_ERR_IO, "open_image: cannot open %s: %s", path, strerror(errno));
  if (fseeko(f.get(), 0, SEEK_END) != 0) return fail(FOXCUDA_ERR_IO, "open_image: cannot size %s", path);
  const uint64_t file_bytes = (uint64_t)ftello(f.get());
  rewind(f.get());
  ImgHeader h;
  if (fread(&h, sizeof h, 1, f.get()) != 1) return fail(FOXCUDA_ERR_FORMAT, "open_image: %s is too short", path);
  if (memcmp(h.magic, kImgMagic, 8) != 0)
    return fail(FOXCUDA_ERR_FORMAT, "open_image: %s is not a foxcuda device image", path);
  if (h.version != kImgVersion)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "open_image: %s has image version %u, this build reads %u", path,
                h.version, kImgVersion);
  if (h.info.n_layer == 0 || h.info.n_layer > 4096 || h.n_entries == 0 || h.n_entries > 16 + 8 * h.info.n_layer)
    return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: %u entries for %u layers", path, h.n_entries, h.info.n_layer);
  const uint64_t head_bytes = sizeof h + (uint64_t)h.n_entries * sizeof(ImgEntry);
  if (h.data_off % 4096 || h.data_off < head_bytes || h.data_off > file_bytes ||
      h.data_bytes != file_bytes - h.data_off)
    return fail(FOXCUDA_ERR_FORMAT, "open_image: %s is truncated or padded (%llu bytes, %llu of data at %llu)",
                path, (unsigned long long)file_bytes, (unsigned long long)h.data_bytes,
                (unsigned long long)h.data_off);
  std::vector<ImgEntry> table(h.n_entries);
  if (fread(table.data(), sizeof(ImgEntry), table.size(), f.get()) != table.size())
    return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: the tensor table is short", path);
  foxcuda_status st = check_image(h, table, path);
  if (st) return st;

  // the device side
  if ((st = foxcuda_init(device))) return st;
  bool any_slice = false;
  for (const ImgEntry& e : table) any_slice |= (e.flags & IMG_SLICE) != 0;
  if (any_slice && h.sm_count != (uint32_t)sm_count(device))
    return fail(FOXCUDA_ERR_UNSUPPORTED, "open_image: %s was laid out for %u SMs and device %d has %d; build the "
                "model from its GGUF here", path, h.sm_count, device, sm_count(device));
  foxcuda_model* m = nullptr;
  if ((st = foxcuda_model_create_tp(&h.info, device, (int)h.tp_rank, (int)h.tp_size, &m))) return st;
  std::unique_ptr<foxcuda_model, void (*)(foxcuda_model*)> guard(m, foxcuda_model_destroy);
  if (memcmp(&m->loc, &h.loc, sizeof h.loc) != 0 || m->vocab0 != h.vocab0 || m->o_block0 != h.o_block0 ||
      m->f_block0 != h.f_block0 || m->f_blocks != h.f_blocks)
    return fail(FOXCUDA_ERR_FORMAT, "open_image: %s: its shard geometry is not this build's", path);
  void* arena = nullptr;
  CK(dev_alloc(m, h.data_bytes, &arena), "open_image: device allocation");
  {
    Staging sg;
    CK(sg.init(2), "open_image staging");
    if (fseeko(f.get(), (off_t)h.data_off, SEEK_SET) != 0) return fail(FOXCUDA_ERR_IO, "open_image: seek in %s", path);
    int i = 0;
    for (uint64_t pos = 0; pos < h.data_bytes; ++i) {
      const int b = i & 1;
      if (i >= 2) CK(cudaEventSynchronize(sg.ev[b]), "open_image copy");  // this buffer's last copy is done
      const size_t n = (size_t)std::min<uint64_t>(kImgChunk, h.data_bytes - pos);
      if (fread(sg.buf[b], 1, n, f.get()) != n) return fail(FOXCUDA_ERR_IO, "open_image: reading %s", path);
      CK(cudaMemcpyAsync((uint8_t*)arena + pos, sg.buf[b], n, cudaMemcpyHostToDevice, sg.s), "open_image copy");
      CK(cudaEventRecord(sg.ev[b], sg.s), "open_image copy");
      pos += n;
    }
    CK(cudaStreamSynchronize(sg.s), "open_image copy");
  }
  uint8_t* base = (uint8_t*)arena;
  uint64_t used = 0;
  auto set_mat = [&](const ImgEntry& e, PackedMat* W) -> foxcuda_status {
    W->type = e.type; W->src_type = e.src_type; W->n_rows = e.n_rows; W->K = e.K; W->nb = e.nb; W->U = e.U;
    W->dev = base + e.offset;
    W->rows32 = (e.flags & IMG_ROWS32) != 0;
    W->pro = e.pro;
    if (e.flags & IMG_SLICE) {
      set_slice(m, W, e.pro);
      if (!W->slice && !W->stream)
        return fail(FOXCUDA_ERR_UNSUPPORTED, "open_image: %s: a slice matrix has no plan on this device", path);
    }
    return FOXCUDA_OK;
  };
  for (const ImgEntry& e : table) {
    used += e.bytes;
    float* fp = reinterpret_cast<float*>(base + e.offset);
    switch (e.kind) {
      case IK_EMBD:
        m->embd.type = e.type; m->embd.src_type = e.src_type; m->embd.ne0 = e.ne0; m->embd.ne1 = e.ne1;
        m->embd.dev = base + e.offset; m->embd.bytes = e.bytes;
        break;
      case IK_OUT_NORM: m->out_norm = fp; break;
      case IK_ATTN_NORM: m->layers[e.layer].attn_norm = fp; break;
      case IK_FFN_NORM: m->layers[e.layer].ffn_norm = fp; break;
      case IK_OUTPUT: st = set_mat(e, &m->output); break;
      case IK_QKV: {
        LayerW& L = m->layers[e.layer];
        st = set_mat(e, &L.qkv[e.index]);
        L.qkv_base[e.index] = e.qkv_base;
        L.n_qkv = (int)e.index + 1;
        break;
      }
      case IK_O: st = set_mat(e, &m->layers[e.layer].o); break;
      case IK_GATEUP: st = set_mat(e, &m->layers[e.layer].gateup); break;
      case IK_DOWN: st = set_mat(e, &m->layers[e.layer].down); break;
      default: break;
    }
    if (st) return st;
  }
  m->device_bytes = used;
  m->finalized = true;
  *out = guard.release();
  return FOXCUDA_OK;
}

// ---------------------------------------------------------------------------
// context

// A pool of K/V pages shared by the contexts of one model: n_pages pages per
// layer, each KV_PAGE positions of every KV head ([kv_head][KV_PAGE][hd]),
// laid out [layer][page]. A paged context takes ceil(n_ctx / KV_PAGE) pages
// at creation and gives them back when destroyed; its block table maps its
// logical pages to them (common.cuh kv_row).
struct foxcuda_kv_pool {
  foxcuda_model* m = nullptr;
  int kv_f16 = 1;
  uint32_t n_pages = 0;
  size_t layer_elems = 0;
  void* k = nullptr;
  void* v = nullptr;
  std::vector<int> free_pages;
  uint32_t users = 0;   // contexts holding pages
  std::mutex mu;
};

struct foxcuda_context {
  foxcuda_model* m = nullptr;
  uint32_t n_ctx = 0;
  int kv_f16 = 1;
  int attn_exact = 0;
  cudaStream_t stream = nullptr;
  float *x = nullptr, *q = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  void *kc = nullptr, *vc = nullptr;
  size_t kv_layer_elems = 0;     // elements between two layers' caches
  int* kv_table = nullptr;       // paged cache: the block table (device), else nullptr
  foxcuda_kv_pool* pool = nullptr;
  std::vector<int> pages;        // this context's pages of the pool, in table order
  int* pos_dev = nullptr;
  uint32_t* token_dev = nullptr;  // [0] the current token, [1] device error code
  int* err_dev = nullptr;
  uint32_t* tokens_dev = nullptr;  // prompt staging
  size_t tokens_cap = 0;
  uint32_t* ring = nullptr;
  float* trace = nullptr;
  bool trace_on = false;
  uint32_t pos = 0;
  cudaGraphExec_t g_body = nullptr, g_full = nullptr;
  uint32_t* h_pinned = nullptr;  // [0] token in, [1..] picks out
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  double last_seconds = 0.0;
  std::vector<void*> allocs;
  std::vector<std::pair<cudaEvent_t, int>>* prof = nullptr;  // diagnostics
  bool tp_steps = false;  // driven through foxcuda_tp_* (collectives between kernels)
  // prompt chunks through the tensor-core pass (foxcuda_context_set_prefill)
  int prefill = 0;
  bool pf_ready = false;
  float *pf_x = nullptr, *pf_xs = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_att = nullptr;
  float *pf_gu = nullptr, *pf_h = nullptr, *pf_t = nullptr;
  int8_t* pf_xq = nullptr;
  int* pf_pos = nullptr;
  // the one-launch attention of a chunk: token t's position pointer, caches
  int** pf_pos_list = nullptr;
  void** pf_k_list = nullptr;
  void** pf_v_list = nullptr;
  float* rows_logits = nullptr;  // foxcuda_eval_all staging, rows_cap x n_vocab
  size_t rows_cap = 0;
  // tensor-parallel exchanges over peer memory (p2p.cuh)
  uint8_t* arena = nullptr;
  size_t terms_d_off = 0;
  int stride_o = 0, stride_d = 0;
  uint8_t* peer_arena[TPX_MAX] = {};
  bool peer_ipc[TPX_MAX] = {};  // mapped through CUDA IPC (closed with the context)
  bool p2p = false;
  float* x_small = nullptr;  // [0..1] global absmax (o, down), [2..3] best pair, [4..] pairs
  unsigned* x_count = nullptr;  // CTAs done of the fused terms / sums GEMV (o, down)
  int x_mode = FOXCUDA_TP_TERMS;  // the row-parallel exchange (foxcuda_tp_p2p_mode)
  size_t y_off = 0;             // the sums area of the arena: [o, down][world][n_embd] words
  // a sums exchange whose residual is not completed yet (which, epoch phase;
  // which < 0: none): the next GEMV over the residual completes it
  int fold_which = -1, fold_phase = 0;
  // repeat penalty of the sharded greedy pick (foxcuda_tp_set_penalty)
  SamplerDev* tp_smp = nullptr;
  float tp_penalty = 1.0f;
};

struct foxcuda_sampler {
  foxcuda_context* c = nullptr;
  foxcuda_sampler_config cfg;
  int k = 0;
  SamplerDev* dev = nullptr;
  cudaGraphExec_t g_decode = nullptr;
  uint32_t n_out = 0;  // host mirror of dev->n_out
};

static cudaError_t ctx_alloc(foxcuda_context* c, size_t bytes, void** p) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e == cudaSuccess) { c->allocs.push_back(*p); cudaMemset(*p, 0, bytes ? bytes : 16); }
  return e;
}

extern "C" void foxcuda_context_destroy(foxcuda_context* c) {
  if (!c) return;
  cudaSetDevice(c->m->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  for (int k = 0; k < TPX_MAX; ++k)
    if (c->peer_arena[k] && c->peer_ipc[k]) cudaIpcCloseMemHandle(c->peer_arena[k]);
  if (c->g_body) cudaGraphExecDestroy(c->g_body);
  if (c->g_full) cudaGraphExecDestroy(c->g_full);
  for (void* p : c->allocs) cudaFree(p);
  if (c->h_pinned) cudaFreeHost(c->h_pinned);
  if (c->ev0) cudaEventDestroy(c->ev0);
  if (c->ev1) cudaEventDestroy(c->ev1);
  if (c->stream) cudaStreamDestroy(c->stream);
  if (c->pool) {
    std::lock_guard<std::mutex> lk(c->pool->mu);
    for (auto it = c->pages.rbegin(); it != c->pages.rend(); ++it) c->pool->free_pages.push_back(*it);
    c->pool->users -= 1;
  }
  delete c;
}

static foxcuda_status context_create(foxcuda_model* m, const foxcuda_context_config* cfg, foxcuda_kv_pool* pool,
                                     foxcuda_context** out) {
  if (!m || !out) return fail(FOXCUDA_ERR_ARG, "context: null argument");
  *out = nullptr;
  if (!m->finalized) {
    foxcuda_status st = foxcuda_model_finalize(m);
    if (st) return st;
  }
  cudaSetDevice(m->device);
  // buffers and kernels use this shard's head and FFN counts
  const foxcuda_model_info& mi = m->loc;
  foxcuda_context* c = new foxcuda_context();
  c->m = m;
  c->n_ctx = cfg && cfg->n_ctx ? cfg->n_ctx : 2048;
  c->kv_f16 = cfg ? cfg->kv_type == FOXCUDA_KV_F16 : 1;
  c->attn_exact = cfg ? cfg->attn_exact != 0 : 0;
  if (c->attn_exact && c->n_ctx > 16384) {
    delete c;
    return fail(FOXCUDA_ERR_UNSUPPORTED, "context: the exact attention mode holds at most 16384 positions");
  }
  const int nq = mi.n_head * mi.head_dim;
  const int half = mi.head_dim / 2;
  const int gqa = mi.n_head / mi.n_head_kv;
  cudaError_t e = cudaSuccess;
  auto A = [&](size_t bytes, void** p) { if (e == cudaSuccess) e = ctx_alloc(c, bytes, p); };
  if (pool) {
    if (pool->m != m || pool->kv_f16 != c->kv_f16) {
      delete c;
      return fail(FOXCUDA_ERR_ARG, "context: the page pool is for another model or cache type");
    }
    const uint32_t need = (c->n_ctx + KV_PAGE - 1) / KV_PAGE;
    {
      std::lock_guard<std::mutex> lk(pool->mu);
      if (pool->free_pages.size() < need) {
        const size_t have = pool->free_pages.size();
        delete c;
        return fail(FOXCUDA_ERR_NOMEM, "context: %u pages needed, %zu free in the pool", need, have);
      }
      for (uint32_t i = 0; i < need; ++i) {
        c->pages.push_back(pool->free_pages.back());
        pool->free_pages.pop_back();
      }
      pool->users += 1;
    }
    c->pool = pool;
    c->kc = pool->k;
    c->vc = pool->v;
    c->kv_layer_elems = pool->layer_elems;
    A(c->pages.size() * sizeof(int), (void**)&c->kv_table);
    if (e == cudaSuccess)
      e = cudaMemcpy(c->kv_table, c->pages.data(), c->pages.size() * sizeof(int), cudaMemcpyHostToDevice);
  } else {
    c->kv_layer_elems = (size_t)mi.n_head_kv * c->n_ctx * mi.head_dim;
    const size_t kv_bytes = c->kv_layer_elems * mi.n_layer * (c->kv_f16 ? 2 : 4);
    A(kv_bytes, &c->kc);
    A(kv_bytes, &c->vc);
  }
  A((size_t)mi.n_embd * 4, (void**)&c->x);
  A((size_t)nq * 4, (void**)&c->q);
  A((size_t)nq * 4, (void**)&c->att);
  A((size_t)mi.n_ff * 4, (void**)&c->h);
  A((size_t)mi.n_vocab * 4, (void**)&c->logits);
  A((size_t)c->n_ctx * half * 4, (void**)&c->rope_cos);
  A((size_t)c->n_ctx * half * 4, (void**)&c->rope_sin);
  A(16, (void**)&c->pos_dev);
  A(16, (void**)&c->token_dev);
  A((size_t)c->n_ctx * 4, (void**)&c->ring);
  if (e == cudaSuccess) {
    c->err_dev = reinterpret_cast<int*>(c->token_dev + 1);
    e = cudaMemset(c->token_dev, 0, 16);
  }
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMallocHost((void**)&c->h_pinned, 64);
  if (e == cudaSuccess) e = cudaEventCreate(&c->ev0);
  if (e == cudaSuccess) e = cudaEventCreate(&c->ev1);
  if (e != cudaSuccess) {
    foxcuda_context_destroy(c);
    return cuda_fail(e, "context allocation");
  }
  // RoPE tables in double, cast to float (upstream src/forward.c:107-118)
  std::vector<float> cs((size_t)c->n_ctx * half), sn((size_t)c->n_ctx * half);
  for (uint32_t p = 0; p < c->n_ctx; ++p)
    for (int i = 0; i < half; ++i) {
      const double th = (double)p * pow((double)mi.rope_freq_base, -2.0 * (double)i / (double)mi.head_dim);
      cs[(size_t)p * half + i] = (float)cos(th);
      sn[(size_t)p * half + i] = (float)sin(th);
    }
  e = cudaMemcpy(c->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(c->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    foxcuda_context_destroy(c);
    return cuda_fail(e, "context init");
  }
  *out = c;
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_context_create(foxcuda_model* m, const foxcuda_context_config* cfg,
                                                 foxcuda_context** out) {
  return context_create(m, cfg, nullptr, out);
}

extern "C" foxcuda_status foxcuda_context_create_paged(foxcuda_model* m, const foxcuda_context_config* cfg,
                                                       foxcuda_kv_pool* pool, foxcuda_context** out) {
  if (!pool) return fail(FOXCUDA_ERR_ARG, "context: null page pool");
  return context_create(m, cfg, pool, out);
}

// The pool's pages are handed out in a fixed shuffled order, so a context's
// pages are scattered over the pool from its first one (the block table is
// what makes them a sequence).
extern "C" foxcuda_status foxcuda_kv_pool_create(foxcuda_model* m, uint32_t n_pages, int kv_type,
                                                 foxcuda_kv_pool** out) {
  if (!m || !out || n_pages == 0) return fail(FOXCUDA_ERR_ARG, "kv_pool: bad argument");
  *out = nullptr;
  if (!m->finalized) {
    foxcuda_status st = foxcuda_model_finalize(m);
    if (st) return st;
  }
  cudaSetDevice(m->device);
  const foxcuda_model_info& mi = m->loc;
  auto pool = std::make_unique<foxcuda_kv_pool>();
  pool->m = m;
  pool->kv_f16 = kv_type == FOXCUDA_KV_F16;
  pool->n_pages = n_pages;
  pool->layer_elems = (size_t)n_pages * mi.n_head_kv * KV_PAGE * mi.head_dim;
  const size_t bytes = pool->layer_elems * mi.n_layer * (pool->kv_f16 ? 2 : 4);
  cudaError_t e = cudaMalloc(&pool->k, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&pool->v, bytes);
  if (e == cudaSuccess) e = cudaMemset(pool->k, 0, bytes);
  if (e == cudaSuccess) e = cudaMemset(pool->v, 0, bytes);
  if (e != cudaSuccess) {
    if (pool->k) cudaFree(pool->k);
    if (pool->v) cudaFree(pool->v);
    return cuda_fail(e, "kv_pool allocation");
  }
  std::vector<int> order(n_pages);
  for (uint32_t i = 0; i < n_pages; ++i) order[i] = (int)i;
  uint64_t st = 0x243F6A8885A308D3ull;
  for (uint32_t i = n_pages - 1; i > 0; --i) {  // Fisher-Yates with a fixed xorshift stream
    st ^= st << 13; st ^= st >> 7; st ^= st << 17;
    std::swap(order[i], order[st % (i + 1)]);
  }
  pool->free_pages.assign(order.rbegin(), order.rend());  // handed out from the back: order[0] first
  *out = pool.release();
  return FOXCUDA_OK;
}

extern "C" uint32_t foxcuda_kv_pool_free_pages(foxcuda_kv_pool* p) {
  if (!p) return 0;
  std::lock_guard<std::mutex> lk(p->mu);
  return (uint32_t)p->free_pages.size();
}

extern "C" foxcuda_status foxcuda_kv_pool_destroy(foxcuda_kv_pool* p) {
  if (!p) return FOXCUDA_OK;
  {
    std::lock_guard<std::mutex> lk(p->mu);
    if (p->users) return fail(FOXCUDA_ERR_ARG, "kv_pool: %u contexts still hold pages", p->users);
  }
  cudaSetDevice(p->m->device);
  cudaFree(p->k);
  cudaFree(p->v);
  delete p;
  return FOXCUDA_OK;
}

extern "C" void foxcuda_context_reset(foxcuda_context* c) {
  if (!c) return;
  cudaSetDevice(c->m->device);
  cudaStreamSynchronize(c->stream);
  c->pos = 0;
  c->fold_which = -1;
  cudaMemsetAsync(c->pos_dev, 0, 4, c->stream);
  cudaStreamSynchronize(c->stream);
}

extern "C" uint32_t foxcuda_context_position(const foxcuda_context* c) { return c ? c->pos : 0; }

// Back to an earlier position: the cache entries from there on are rewritten
// by the next tokens (speculative decoding drops the rejected draft so).
extern "C" foxcuda_status foxcuda_context_rewind(foxcuda_context* c, uint32_t pos) {
  if (!c) return fail(FOXCUDA_ERR_ARG, "rewind: null context");
  if (pos > c->pos) return fail(FOXCUDA_ERR_ARG, "rewind: position %u is past the current %u", pos, c->pos);
  // Peer-memory exchange slots are tagged with the position they serve: a
  // replayed position would accept a peer's stale value as this step's.
  if (c->p2p && pos != c->pos)
    return fail(FOXCUDA_ERR_ARG, "rewind: not supported on a context with peer-memory exchanges "
                "(reset every shard and clear its arena instead)");
  cudaSetDevice(c->m->device);
  CK(cudaStreamSynchronize(c->stream), "rewind");
  const int p = (int)pos;
  CK(cudaMemcpy(c->pos_dev, &p, 4, cudaMemcpyHostToDevice), "rewind");
  c->pos = pos;
  return FOXCUDA_OK;
}
extern "C" double foxcuda_context_last_eval_seconds(const foxcuda_context* c) {
  return c ? c->last_seconds : 0.0;
}

// One token through the layers (upstream src/forward.c:315-399): embedding,
// then per layer the fused q|k|v (+RMSNorm, +RoPE, +KV write), attention, o
// (+residual), gate|up (+RMSNorm, +SwiGLU), down (+residual); pos += 1.
// Launch kinds of a decode step (diagnostics name them by these numbers).
enum { PK_EMBED = 0, PK_QKV, PK_ATTN, PK_O, PK_GATEUP, PK_DOWN, PK_ADVANCE, PK_HEAD, PK_PICK };

// While a context is being profiled an event follows every launch.
static void mark(foxcuda_context* c, int kind);
// tensor-parallel sums exchange: the residual completed before a GEMV over
// it, by a kernel of its own or in the GEMV's prologue
static cudaError_t enqueue_fold(foxcuda_context* c);
static void set_nfold(const foxcuda_context* c, GemvParams& p);
static foxcuda_status flush_fold(foxcuda_context* c) {
  CK(enqueue_fold(c), "tp sums fold");
  return FOXCUDA_OK;
}

static void* kv_layer(const foxcuda_context* c, void* base, uint32_t l) {
  return (uint8_t*)base + (size_t)l * c->kv_layer_elems * (c->kv_f16 ? 2 : 4);
}


// Weight bytes (GGUF bytes) of one launch of a layer kernel, 0 for others.
static uint64_t gguf_bytes(const PackedMat& W) {
  return (uint64_t)W.n_rows * row_bytes(W.src_type >= 0 ? W.src_type : W.type, W.K);
}

static uint64_t launch_weight_bytes(const foxcuda_model* m, int kind, uint32_t l) {
  const LayerW& L = m->layers[l];
  switch (kind) {
    case PK_QKV: { uint64_t b = 0; for (int i = 0; i < L.n_qkv; ++i) b += gguf_bytes(L.qkv[i]); return b; }
    case PK_O: return gguf_bytes(L.o);
    case PK_GATEUP: return gguf_bytes(L.gateup);
    case PK_DOWN: return gguf_bytes(L.down);
    case PK_HEAD: return gguf_bytes(m->output);
    default: return 0;
  }
}


// Whether the context's GEMVs, attention and head overlap their
// predecessors (programmatic stream serialisation): the single-GPU step, and
// a tensor-parallel step whose exchanges run over peer memory (its stream
// holds only this library's kernels). A tensor-parallel step with NCCL
// collectives between its kernels keeps plain stream order: a kernel
// overlapped after one of those read its input before it landed (measured:
// the head after the last fold, with the collective on the process group's
// own stream, joined by an event).
static bool ctx_pdl(const foxcuda_context* c) {
  if (c->m->tp_size == 1 && !c->tp_steps) return true;
  return c->p2p;
}

// A layer GEMV through the kernel its layout was packed for.
static cudaError_t launch_mat(foxcuda_context* c, const PackedMat& W, int pro, int epi, GemvParams& p) {
  p.err = c->err_dev;
  p.pdl = ctx_pdl(c);
  if (W.slice || W.stream) return launch_sliced(W, pro, epi, p, c->stream);
  return launch_ring(W.type, pro, epi, p, c->stream);
}

// The fused q|k|v GEMV(s) of layer l: RMSNorm + quantise prologue, RoPE and
// K/V cache write epilogue.
static cudaError_t launch_qkv(foxcuda_context* c, uint32_t l) {
  const foxcuda_model_info& mi = c->m->info;
  const LayerW& L = c->m->layers[l];
  // a pending sums exchange: one fused matrix completes the residual in its
  // prologue; runs of several types take the sum as a kernel first
  const bool fold = c->fold_which >= 0 && L.n_qkv == 1;
  if (c->fold_which >= 0 && !fold) {
    cudaError_t e = enqueue_fold(c);
    if (e) return e;
  }
  for (int i = 0; i < L.n_qkv; ++i) {
    const PackedMat& W = L.qkv[i];
    GemvParams p = gemv_base(W.type, W.dev, W.n_rows, W.K, W.nb, W.U);
    p.x = c->x; p.norm_w = L.attn_norm; p.eps = mi.rms_eps;
    p.out = c->q; p.nq = c->m->loc.n_head * mi.head_dim; p.nkv = c->m->loc.n_head_kv * mi.head_dim;
    p.hd = mi.head_dim; p.n_ctx = c->n_ctx; p.kv_f16 = c->kv_f16;
    p.rope_cos = c->rope_cos; p.rope_sin = c->rope_sin; p.pos = c->pos_dev;
    p.kcache = kv_layer(c, c->kc, l); p.vcache = kv_layer(c, c->vc, l); p.row_base = L.qkv_base[i];
    p.kv_table = c->kv_table;
    if (fold) set_nfold(c, p);
    cudaError_t e = launch_mat(c, W, fold ? PRO_NFOLD : PRO_NORM, EPI_QKV, p);
    if (e) return e;
  }
  if (fold) c->fold_which = -1;
  return cudaSuccess;
}

// The tile attention (attn.cuh) of n_seq sequences in one launch: grid
// (nt, n_kv, n_seq) in clusters of nt CTAs. pdl: launched with programmatic
// stream serialisation, right after the kernel that writes q and the newest
// K/V row and nothing else this kernel reads (the decode step's q|k|v GEMV).
template <int DPL, bool F16, int G>
static cudaError_t launch_tile_g(const AttnParams& ap_in, int n_seq, cudaStream_t s, bool pdl) {
  auto kern = attention_tile_kernel<DPL, F16, G>;
  AttnParams ap = ap_in;
  attn_ring(ap, G);
  const size_t sm = attn_tile_smem_bytes(ap.n_ctx, ap.nt, G, ap.hd, F16 ? 1 : 0, ap.stage_rows, ap.stage_slots);
  static size_t marks[kMaxDevices] = {};
  cudaError_t e = opt_in_smem(kern, sm, marks);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ap.nt, ap.n_kv, n_seq);
  cfg.blockDim = dim3(ATTN_THREADS);
  cfg.dynamicSmemBytes = sm;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = ap.nt;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, ap);
}

template <int DPL, bool F16>
static cudaError_t launch_tile_f(const AttnParams& ap, int n_seq, cudaStream_t s, bool pdl) {
  switch (ap.n_head / ap.n_kv) {
    case 1: return launch_tile_g<DPL, F16, 1>(ap, n_seq, s, pdl);
    case 2: return launch_tile_g<DPL, F16, 2>(ap, n_seq, s, pdl);
    case 4: return launch_tile_g<DPL, F16, 4>(ap, n_seq, s, pdl);
    case 8: return launch_tile_g<DPL, F16, 8>(ap, n_seq, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <int DPL>
static cudaError_t launch_tile_t(const AttnParams& ap, int n_seq, cudaStream_t s, bool pdl) {
  return ap.kv_f16 ? launch_tile_f<DPL, true>(ap, n_seq, s, pdl) : launch_tile_f<DPL, false>(ap, n_seq, s, pdl);
}

static cudaError_t launch_tiles(const AttnParams& ap, int n_seq, cudaStream_t s, bool pdl = false) {
  switch (ap.hd / 32) {
    case 2: return launch_tile_t<2>(ap, n_seq, s, pdl);
    case 4: return launch_tile_t<4>(ap, n_seq, s, pdl);
    case 8: return launch_tile_t<8>(ap, n_seq, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

// One decode attention over a K/V cache: upstream's serial order (exact) or
// the tile attention.
static cudaError_t run_attention(const AttnParams& ap, bool exact, cudaStream_t s, bool pdl) {
  if (!exact) return launch_tiles(ap, 1, s, pdl);
  const size_t sm = (size_t)ap.n_ctx * 4;
  static size_t marks[kMaxDevices] = {};
  cudaError_t e = opt_in_smem(attention_exact_kernel, sm, marks);
  if (e != cudaSuccess) return e;
  attention_exact_kernel<<<ap.n_head, 128, sm, s>>>(ap);
  return cudaGetLastError();
}

static cudaError_t launch_attn(foxcuda_context* c, uint32_t l) {
  const foxcuda_model_info& mi = c->m->info;
  AttnParams ap{};
  ap.q = c->q; ap.kcache = kv_layer(c, c->kc, l); ap.vcache = kv_layer(c, c->vc, l); ap.kv_table = c->kv_table;
  ap.kv_f16 = c->kv_f16; ap.n_ctx = c->n_ctx;
  ap.hd = mi.head_dim; ap.n_head = c->m->loc.n_head; ap.n_kv = c->m->loc.n_head_kv; ap.nt = c->m->attn_nt;
  ap.pos = c->pos_dev; ap.out = c->att;
  ap.scale = 1.0f / sqrtf((float)mi.head_dim);
  return run_attention(ap, c->attn_exact, c->stream, ctx_pdl(c));
}

static cudaError_t launch_o(foxcuda_context* c, uint32_t l) {
  const PackedMat& W = c->m->layers[l].o;
  GemvParams p = gemv_base(W.type, W.dev, W.n_rows, W.K, W.nb, W.U);
  p.x = c->att; p.out = c->x;
  return launch_mat(c, W, PRO_VEC, EPI_ADD, p);
}

static cudaError_t launch_gateup(foxcuda_context* c, uint32_t l) {
  const LayerW& L = c->m->layers[l];
  const PackedMat& W = L.gateup;
  GemvParams p = gemv_base(W.type, W.dev, W.n_rows, W.K, W.nb, W.U);
  p.x = c->x; p.norm_w = L.ffn_norm; p.eps = c->m->info.rms_eps; p.out = c->h;
  if (c->fold_which < 0) return launch_mat(c, W, PRO_NORM, EPI_SWIGLU, p);
  set_nfold(c, p);  // completes the pending sums exchange in its prologue
  c->fold_which = -1;
  return launch_mat(c, W, PRO_NFOLD, EPI_SWIGLU, p);
}

static cudaError_t launch_down(foxcuda_context* c, uint32_t l) {
  const PackedMat& W = c->m->layers[l].down;
  GemvParams p = gemv_base(W.type, W.dev, W.n_rows, W.K, W.nb, W.U);
  p.x = c->h; p.out = c->x;
  return launch_mat(c, W, PRO_VEC, EPI_ADD, p);
}

// One block of look-ahead per warp: two (twice the bytes in flight at the
// same occupancy) measured the same, 661 against 661 tok/s for the 4B step.
static cudaError_t launch_q8_rows(const GemvParams& p, cudaStream_t s) {
  auto kern = q8_rows_kernel<PRO_NORM, 1>;
  const size_t smem = (size_t)p.K * 4 + 32 * 8;
  static size_t marks[kMaxDevices] = {};  // one kernel per process (the variable is read once)
  cudaError_t e = opt_in_smem(kern, smem, marks);
  if (e != cudaSuccess) return e;
  const int pairs = (p.n_rows / 32 + 1) / 2;
  const int warps = ROWS_THREADS / 32;
  const int grid = std::max(1, std::min((pairs + warps - 1) / warps, 4 * current_sms()));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(ROWS_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

// Output norm on the last token and the head (upstream src/forward.c:403-408).
static cudaError_t launch_head_on(foxcuda_context* c, cudaStream_t s, bool pdl) {
  foxcuda_model* m = c->m;
  const PackedMat& H = m->output;
  GemvParams p = gemv_base(H.type, H.dev, H.n_rows, H.K, H.nb, H.U);
  p.x = c->x; p.norm_w = m->out_norm; p.eps = m->info.rms_eps; p.out = c->logits;
  p.err = c->err_dev;
  p.pdl = pdl;
  if (H.rows32) return launch_q8_rows(p, s);
  return launch_ring(H.type, PRO_NORM, EPI_STORE, p, s);
}

static cudaError_t launch_head(foxcuda_context* c) { return launch_head_on(c, c->stream, ctx_pdl(c)); }

static cudaError_t enqueue_body(foxcuda_context* c, bool trace) {
  foxcuda_model* m = c->m;
  const foxcuda_model_info& mi = m->info;
  cudaStream_t s = c->stream;
  const size_t emb_rb = row_bytes(m->embd.type, mi.n_embd);
  embed_kernel<<<(mi.n_embd + 255) / 256, 256, 0, s>>>(m->embd.type, m->embd.dev, emb_rb,
                                                        (int)mi.n_embd, c->token_dev, c->x);
  cudaError_t e = cudaGetLastError();
  if (e) return e;
  mark(c, PK_EMBED);
  if (trace) cudaMemcpyAsync(c->trace, c->x, mi.n_embd * 4, cudaMemcpyDeviceToDevice, s);
  for (uint32_t l = 0; l < mi.n_layer; ++l) {
    if ((e = launch_qkv(c, l))) return e;
    mark(c, PK_QKV);
    if ((e = launch_attn(c, l))) return e;
    mark(c, PK_ATTN);
    if ((e = launch_o(c, l))) return e;
    mark(c, PK_O);
    if ((e = launch_gateup(c, l))) return e;
    mark(c, PK_GATEUP);
    if ((e = launch_down(c, l))) return e;
    mark(c, PK_DOWN);
    if (trace) cudaMemcpyAsync(c->trace + (size_t)(l + 1) * mi.n_embd, c->x, mi.n_embd * 4,
                               cudaMemcpyDeviceToDevice, s);
  }
  advance_kernel<<<1, 32, 0, s>>>(c->pos_dev, 1);
  mark(c, PK_ADVANCE);
  return cudaGetLastError();
}

static cudaError_t enqueue_head(foxcuda_context* c) {
  cudaError_t e = launch_head(c);
  mark(c, PK_HEAD);
  return e;
}

static cudaError_t enqueue_pick_on(foxcuda_sampler* sm, bool accept, cudaStream_t s) {
  foxcuda_context* c = sm->c;
  const int nv = c->m->info.n_vocab;
  const bool pen = sm->cfg.repeat_penalty > 1.0f;
  if (pen) penalty_kernel<<<1, 256, 0, s>>>(sm->dev, c->logits, nv, sm->cfg.repeat_penalty);
  if (sm->cfg.temperature <= 0.0f) {
    const int grid = std::min(1024, std::max(1, std::min(current_sms(), (nv + ARGMAX_THREADS - 1) / ARGMAX_THREADS)));
    argmax_kernel<<<grid, ARGMAX_THREADS, 0, s>>>(sm->dev, c->logits, nv, pen, accept,
                                                   c->token_dev, c->ring, (int)c->n_ctx);
  } else {
    topk_sample_kernel<<<1, TOPK_THREADS, 0, s>>>(sm->dev, c->logits, nv, sm->k,
                                                  sm->cfg.temperature, sm->cfg.top_p, pen,
                                                  accept, c->token_dev, c->ring,
                                                  (int)c->n_ctx);
  }
  return cudaGetLastError();
}

static cudaError_t enqueue_pick(foxcuda_sampler* sm, bool accept) {
  cudaError_t e = enqueue_pick_on(sm, accept, sm->c->stream);
  mark(sm->c, PK_PICK);
  return e;
}

static cudaError_t capture(foxcuda_context* c, cudaGraphExec_t* out, bool head, foxcuda_sampler* sm) {
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal);
  if (e) return e;
  e = enqueue_body(c, false);
  if (!e && head) e = enqueue_head(c);
  if (!e && sm) e = enqueue_pick(sm, true);
  cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
  if (e) { if (g) cudaGraphDestroy(g); return e; }
  if (e2) return e2;
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  return e;
}


extern "C" foxcuda_status foxcuda_context_set_trace(foxcuda_context* c, int on) {
  if (!c) return fail(FOXCUDA_ERR_ARG, "trace: null context");
  cudaSetDevice(c->m->device);
  if (on && !c->trace) {
    void* p = nullptr;
    CK(ctx_alloc(c, (size_t)(c->m->info.n_layer + 1) * c->m->info.n_embd * 4, &p), "trace alloc");
    c->trace = (float*)p;
  }
  c->trace_on = on != 0;
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_context_hidden(const foxcuda_context* c, uint32_t layer, float* out) {
  if (!c || !out) return fail(FOXCUDA_ERR_ARG, "hidden: null argument");
  if (!c->trace) return fail(FOXCUDA_ERR_ARG, "hidden: tracing is off");
  if (layer > c->m->info.n_layer) return fail(FOXCUDA_ERR_ARG, "hidden: layer %u out of range", layer);
  cudaSetDevice(c->m->device);
  CK(cudaMemcpy(out, c->trace + (size_t)layer * c->m->info.n_embd, c->m->info.n_embd * 4,
                cudaMemcpyDeviceToHost), "hidden copy");
  return FOXCUDA_OK;
}

// A bounded device wait that gave up leaves a nonzero code in err_dev. The
// code is copied to h_pinned[3] before each synchronising call returns and
// reported here; the flag is cleared for the next step.
static void enqueue_err_read(foxcuda_context* c) {
  cudaMemcpyAsync(c->h_pinned + 3, c->err_dev, 4, cudaMemcpyDeviceToHost, c->stream);
}

static foxcuda_status check_err(foxcuda_context* c) {
  const uint32_t code = c->h_pinned[3];
  if (!code) return FOXCUDA_OK;
  c->h_pinned[3] = 0;
  cudaMemsetAsync(c->err_dev, 0, 4, c->stream);
  cudaStreamSynchronize(c->stream);
  return fail(FOXCUDA_ERR_INTERNAL, "device: a bounded wait gave up (code %u: 1 weights to shared memory, "
              "2 a peer's exchange); the step's outputs are not valid", code);
}

// ---------------------------------------------------------------------------
// prompt chunks through the tensor-core pass (prefill.cuh, tc.cuh)

constexpr int PF_CHUNK = 64;  // tokens per chunk: the widest token tile of the pass

// Threads of the decode kernel that normalises W's input vector: the chunk
// forms its double sums of squares in the same partition.
static int decode_threads(const PackedMat& W) {
  return W.slice ? SLICE_THREADS : W.stream ? STREAM_THREADS : (W.U * W.nb + 31) / 32 * 32;
}

// Every layer matrix can take the tensor-core pass (ternary, held as TQ2_0)
// and the row kernels (inputs of at most 200 KB of floats).
static bool tc_layers_ok(const foxcuda_model* m) {
  if (m->tp_size != 1) return false;
  for (const LayerW& L : m->layers) {
    if (L.n_qkv != 1) return false;
    for (const PackedMat* W : {&L.qkv[0], &L.o, &L.gateup, &L.down})
      if (W->type != T_TQ2_0 || W->nb > TC_MAX_NB || (size_t)W->K * 4 > 200 * 1024) return false;
  }
  return true;
}

static bool prefill_eligible(const foxcuda_context* c) {
  return c->prefill && !c->trace_on && tc_layers_ok(c->m);
}

static cudaError_t prefill_buffers(foxcuda_context* c) {
  if (c->pf_ready) return cudaSuccess;
  const foxcuda_model_info& mi = c->m->loc;
  const size_t E = mi.n_embd, nq = (size_t)mi.n_head * mi.head_dim, nkv = (size_t)mi.n_head_kv * mi.head_dim;
  const size_t F = mi.n_ff, M = PF_CHUNK;
  const size_t kmax = std::max(E, std::max(nq, F));
  cudaError_t e = cudaSuccess;
  auto A = [&](size_t bytes, void** p) { if (e == cudaSuccess) e = ctx_alloc(c, bytes, p); };
  A(M * E * 4, (void**)&c->pf_x);
  A(M * kmax, (void**)&c->pf_xq);
  A(M * (kmax / 256 + 1) * 4, (void**)&c->pf_xs);  // one scale per token, or per 256 block (K-quants)
  A(M * (nq + 2 * nkv) * 4, (void**)&c->pf_qkv);
  A(M * nq * 4, (void**)&c->pf_q);
  A(M * nq * 4, (void**)&c->pf_att);
  A(M * 2 * F * 4, (void**)&c->pf_gu);
  A(M * F * 4, (void**)&c->pf_h);
  A(M * E * 4, (void**)&c->pf_t);
  A(M * 4, (void**)&c->pf_pos);
  A(M * sizeof(int*), (void**)&c->pf_pos_list);
  A(M * sizeof(void*), (void**)&c->pf_k_list);
  A(M * sizeof(void*), (void**)&c->pf_v_list);
  if (e == cudaSuccess) {
    std::vector<int*> pl(M);
    std::vector<void*> kl(M, c->kc), vl(M, c->vc);
    for (size_t t = 0; t < M; ++t) pl[t] = c->pf_pos + t;
    e = cudaMemcpy(c->pf_pos_list, pl.data(), M * sizeof(int*), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(c->pf_k_list, kl.data(), M * sizeof(void*), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(c->pf_v_list, vl.data(), M * sizeof(void*), cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) c->pf_ready = true;
  return e;
}

template <bool NORM>
static cudaError_t quant_rows_to(const float* X, int K, const float* norm_w, float eps, int threads, int M,
                                 int8_t* XQ, float* XS, cudaStream_t s) {
  const size_t smem = (size_t)K * 4;
  static size_t marks[kMaxDevices] = {};
  cudaError_t e = opt_in_smem(quant_rows_kernel<NORM>, smem, marks);
  if (e != cudaSuccess) return e;
  quant_rows_kernel<NORM><<<M, threads, smem, s>>>(X, K, norm_w, eps, XQ, XS);
  return cudaGetLastError();
}

template <bool NORM>
static cudaError_t quant_rows(foxcuda_context* c, const float* X, int K, const float* norm_w, int threads,
                              int M) {
  return quant_rows_to<NORM>(X, K, norm_w, c->m->info.rms_eps, threads, M, c->pf_xq, c->pf_xs, c->stream);
}

// out[t][r] for M quantised rows through W (TQ2_0, packed)
static cudaError_t tc_rows_to(const int8_t* XQ, const float* XS, const PackedMat& W, int M, float* out, int* err,
                              cudaStream_t s) {
  TcParams p = tc_params(XQ, XS, (size_t)M, W.dev, (size_t)W.n_rows, (size_t)W.K, W.U, out);
  p.err = err;
  return launch_tc(p, s);
}

static cudaError_t tc_rows(foxcuda_context* c, const PackedMat& W, int M, float* out) {
  return tc_rows_to(c->pf_xq, c->pf_xs, W, M, out, c->err_dev, c->stream);
}

// Layer l's attention of every token of a chunk over positions 0..its own
// (its K/V rows and the chunk's later ones are in the cache already; each
// token reads only up to its own position). one_launch takes the cluster
// kernel with grid z = token, every token naming the same caches; otherwise
// one decode attention launch per token. Both give the decode step's values.
static cudaError_t chunk_attention(foxcuda_context* c, uint32_t l, int M, bool one_launch) {
  const foxcuda_model* m = c->m;
  const int hd = m->info.head_dim, nq = m->loc.n_head * hd;
  AttnParams ap{};
  ap.kv_f16 = c->kv_f16; ap.n_ctx = c->n_ctx;
  ap.hd = hd; ap.n_head = m->loc.n_head; ap.n_kv = m->loc.n_head_kv; ap.nt = m->attn_nt;
  ap.scale = 1.0f / sqrtf((float)hd);
  if (one_launch && !c->attn_exact) {
    ap.q = c->pf_q; ap.out = c->pf_att; ap.seq_stride = nq;
    ap.pos_list = c->pf_pos_list; ap.k_list = c->pf_k_list; ap.v_list = c->pf_v_list;
    ap.layer_off = (size_t)l * c->kv_layer_elems * (c->kv_f16 ? 2 : 4);
    return launch_tiles(ap, M, c->stream);
  }
  ap.kcache = kv_layer(c, c->kc, l); ap.vcache = kv_layer(c, c->vc, l); ap.kv_table = c->kv_table;
  cudaError_t e = cudaSuccess;
  for (int t = 0; t < M && !e; ++t) {
    ap.q = c->pf_q + (size_t)t * nq;
    ap.pos = c->pf_pos + t;
    ap.out = c->pf_att + (size_t)t * nq;
    e = run_attention(ap, c->attn_exact, c->stream);
  }
  return e;
}

// M prompt tokens (device ids) at positions pos0.. through every layer; the
// last one's residual row is left in c->x for the head, and the device
// position moves past the chunk. Per token the values are the decode step's.
static cudaError_t prefill_chunk(foxcuda_context* c, const uint32_t* tokens, int M, uint32_t pos0,
                                 bool one_launch) {
  foxcuda_model* m = c->m;
  const foxcuda_model_info& mi = m->info;
  cudaStream_t s = c->stream;
  const int E = mi.n_embd, hd = mi.head_dim;
  const int nq = m->loc.n_head * hd, nkv = m->loc.n_head_kv * hd, F = m->loc.n_ff, nqkv = nq + 2 * nkv;
  const size_t rows_e = (size_t)M * E;
  const unsigned add_grid = (unsigned)std::min<size_t>((rows_e + 255) / 256, 4096);
  embed_rows_kernel<<<dim3((E + 255) / 256, M), 256, 0, s>>>(m->embd.type, m->embd.dev,
                                                            row_bytes(m->embd.type, E), E, tokens, c->pf_x);
  positions_kernel<<<(M + 127) / 128, 128, 0, s>>>(c->pf_pos, (int)pos0, M);
  cudaError_t e = cudaGetLastError();
  for (uint32_t l = 0; l < mi.n_layer && !e; ++l) {
    const LayerW& L = m->layers[l];
    // q|k|v, RoPE, K/V of every token of the chunk
    if ((e = quant_rows<true>(c, c->pf_x, E, L.attn_norm, decode_threads(L.qkv[0]), M))) break;
    if ((e = tc_rows(c, L.qkv[0], M, c->pf_qkv))) break;
    qkv_rows_kernel<<<dim3((nqkv + 255) / 256, M), 256, 0, s>>>(
        c->pf_qkv, nqkv, nq, nkv, hd, (int)c->n_ctx, (int)pos0, c->rope_cos, c->rope_sin, c->kv_f16,
        kv_layer(c, c->kc, l), kv_layer(c, c->vc, l), c->kv_table, c->pf_q);
    if ((e = cudaGetLastError())) break;
    if ((e = chunk_attention(c, l, M, one_launch))) break;
    // o, residual
    if ((e = quant_rows<false>(c, c->pf_att, nq, nullptr, 256, M))) break;
    if ((e = tc_rows(c, L.o, M, c->pf_t))) break;
    add_rows_kernel<<<add_grid, 256, 0, s>>>(c->pf_x, c->pf_t, rows_e);
    // gate|up, SwiGLU
    if ((e = quant_rows<true>(c, c->pf_x, E, L.ffn_norm, decode_threads(L.gateup), M))) break;
    if ((e = tc_rows(c, L.gateup, M, c->pf_gu))) break;
    swiglu_rows_kernel<<<dim3((F + 255) / 256, M), 256, 0, s>>>(c->pf_gu, 2 * F, L.gateup.U, c->pf_h);
    // down, residual
    if ((e = quant_rows<false>(c, c->pf_h, F, nullptr, 256, M))) break;
    if ((e = tc_rows(c, L.down, M, c->pf_t))) break;
    add_rows_kernel<<<add_grid, 256, 0, s>>>(c->pf_x, c->pf_t, rows_e);
    e = cudaGetLastError();
  }
  if (e) return e;
  if ((e = cudaMemcpyAsync(c->x, c->pf_x + (size_t)(M - 1) * E, (size_t)E * 4, cudaMemcpyDeviceToDevice, s)))
    return e;
  if ((e = cudaMemcpyAsync(c->token_dev, tokens + M - 1, 4, cudaMemcpyDeviceToDevice, s))) return e;
  advance_kernel<<<1, 32, 0, s>>>(c->pos_dev, M);
  return cudaGetLastError();
}

// ---- the same chunk for K-quant models (tc_kquant.cuh) ----------------------

static bool is_kq(int t) { return t == T_Q4_K || t == T_Q6_K; }

// Every layer matrix is Q4_K or Q6_K with inputs of at most 200 KB of floats.
static bool kq_layers_ok(const foxcuda_model* m) {
  if (m->tp_size != 1) return false;
  for (const LayerW& L : m->layers) {
    for (int i = 0; i < L.n_qkv; ++i)
      if (!is_kq(L.qkv[i].type)) return false;
    for (const PackedMat* W : {&L.o, &L.gateup, &L.down})
      if (!is_kq(W->type) || (size_t)W->K * 4 > 200 * 1024) return false;
  }
  return (size_t)m->info.n_embd * 4 <= 200 * 1024;
}

template <bool NORM>
static cudaError_t quant_rows_k_to(const float* X, int K, const float* norm_w, float eps, int threads, int M,
                                   int8_t* XQ, float* XS, cudaStream_t s) {
  const size_t smem = (size_t)K * 4;
  static size_t marks[kMaxDevices] = {};
  cudaError_t e = opt_in_smem(quant_rows_k_kernel<NORM>, smem, marks);
  if (e != cudaSuccess) return e;
  quant_rows_k_kernel<NORM><<<M, threads, smem, s>>>(X, K, norm_w, eps, XQ, XS);
  return cudaGetLastError();
}

template <bool NORM>
static cudaError_t quant_rows_k(foxcuda_context* c, const float* X, int K, const float* norm_w, int threads,
                                int M) {
  return quant_rows_k_to<NORM>(X, K, norm_w, c->m->info.rms_eps, threads, M, c->pf_xq, c->pf_xs, c->stream);
}

static cudaError_t kq_rows_to(const int8_t* XQ, const float* XS, const PackedMat& W, int M, float* out,
                              int out_stride, int* err, cudaStream_t s) {
  TcKParams p;
  p.w = W.dev; p.xq = XQ; p.xs = XS; p.out = out; p.out_stride = out_stride;
  p.n_rows = W.n_rows; p.K = W.K; p.nb = W.K / 256; p.U = W.U; p.n_tok = M; p.err = err;
  return launch_kq(W.type, p, s);
}

static cudaError_t kq_rows(foxcuda_context* c, const PackedMat& W, int M, float* out, int out_stride) {
  return kq_rows_to(c->pf_xq, c->pf_xs, W, M, out, out_stride, c->err_dev, c->stream);
}

// prefill_chunk for K-quant layers: each q|k|v run is quantised with the
// thread count of its own decode kernel and lands at its row offset.
static cudaError_t prefill_chunk_kq(foxcuda_context* c, const uint32_t* tokens, int M, uint32_t pos0,
                                    bool one_launch) {
  foxcuda_model* m = c->m;
  const foxcuda_model_info& mi = m->info;
  cudaStream_t s = c->stream;
  const int E = mi.n_embd, hd = mi.head_dim;
  const int nq = m->loc.n_head * hd, nkv = m->loc.n_head_kv * hd, F = m->loc.n_ff, nqkv = nq + 2 * nkv;
  const size_t rows_e = (size_t)M * E;
  const unsigned add_grid = (unsigned)std::min<size_t>((rows_e + 255) / 256, 4096);
  embed_rows_kernel<<<dim3((E + 255) / 256, M), 256, 0, s>>>(m->embd.type, m->embd.dev,
                                                            row_bytes(m->embd.type, E), E, tokens, c->pf_x);
  positions_kernel<<<(M + 127) / 128, 128, 0, s>>>(c->pf_pos, (int)pos0, M);
  cudaError_t e = cudaGetLastError();
  for (uint32_t l = 0; l < mi.n_layer && !e; ++l) {
    const LayerW& L = m->layers[l];
    for (int i = 0; i < L.n_qkv && !e; ++i) {
      if ((e = quant_rows_k<true>(c, c->pf_x, E, L.attn_norm, decode_threads(L.qkv[i]), M))) break;
      e = kq_rows(c, L.qkv[i], M, c->pf_qkv + L.qkv_base[i], nqkv);
    }
    if (e) break;
    qkv_rows_kernel<<<dim3((nqkv + 255) / 256, M), 256, 0, s>>>(
        c->pf_qkv, nqkv, nq, nkv, hd, (int)c->n_ctx, (int)pos0, c->rope_cos, c->rope_sin, c->kv_f16,
        kv_layer(c, c->kc, l), kv_layer(c, c->vc, l), c->kv_table, c->pf_q);
    if ((e = cudaGetLastError())) break;
    if ((e = chunk_attention(c, l, M, one_launch))) break;
    if ((e = quant_rows_k<false>(c, c->pf_att, nq, nullptr, 256, M))) break;
    if ((e = kq_rows(c, L.o, M, c->pf_t, E))) break;
    add_rows_kernel<<<add_grid, 256, 0, s>>>(c->pf_x, c->pf_t, rows_e);
    if ((e = quant_rows_k<true>(c, c->pf_x, E, L.ffn_norm, decode_threads(L.gateup), M))) break;
    if ((e = kq_rows(c, L.gateup, M, c->pf_gu, 2 * F))) break;
    swiglu_rows_kernel<<<dim3((F + 255) / 256, M), 256, 0, s>>>(c->pf_gu, 2 * F, L.gateup.U, c->pf_h);
    if ((e = quant_rows_k<false>(c, c->pf_h, F, nullptr, 256, M))) break;
    if ((e = kq_rows(c, L.down, M, c->pf_t, E))) break;
    add_rows_kernel<<<add_grid, 256, 0, s>>>(c->pf_x, c->pf_t, rows_e);
    e = cudaGetLastError();
  }
  if (e) return e;
  if ((e = cudaMemcpyAsync(c->x, c->pf_x + (size_t)(M - 1) * E, (size_t)E * 4, cudaMemcpyDeviceToDevice, s)))
    return e;
  if ((e = cudaMemcpyAsync(c->token_dev, tokens + M - 1, 4, cudaMemcpyDeviceToDevice, s))) return e;
  advance_kernel<<<1, 32, 0, s>>>(c->pos_dev, M);
  return cudaGetLastError();
}

extern "C" foxcuda_status foxcuda_context_set_prefill(foxcuda_context* c, int mode) {
  if (!c || (mode != 0 && mode != 1)) return fail(FOXCUDA_ERR_ARG, "set_prefill: mode is 0 or 1");
  c->prefill = mode;
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_eval(foxcuda_context* c, const uint32_t* tokens, size_t n,
                                       float* logits_out) {
  if (!c || !tokens || n == 0) return fail(FOXCUDA_ERR_ARG, "eval: nothing to evaluate");
  if (c->m->tp_size > 1)
    return fail(FOXCUDA_ERR_ARG, "eval: a tensor-parallel shard decodes through foxcuda_tp_*");
  const foxcuda_model_info& mi = c->m->info;
  if ((size_t)c->pos + n > c->n_ctx)
    return fail(FOXCUDA_ERR_ARG, "forward: %zu tokens past position %u would overrun the %u token context",
                n, c->pos, c->n_ctx);
  for (size_t i = 0; i < n; ++i)
    if (tokens[i] >= mi.n_vocab)
      return fail(FOXCUDA_ERR_ARG, "forward: token %u is outside the %u entry vocabulary", tokens[i], mi.n_vocab);
  cudaSetDevice(c->m->device);
  if (n > c->tokens_cap) {
    void* p = nullptr;
    CK(ctx_alloc(c, n * 4, &p), "token staging");
    c->tokens_dev = (uint32_t*)p;
    c->tokens_cap = n;
  }
  CK(cudaMemcpyAsync(c->tokens_dev, tokens, n * 4, cudaMemcpyHostToDevice, c->stream), "token upload");
  if (!c->trace_on && !c->g_body) CK(capture(c, &c->g_body, false, nullptr), "capture");
  if (!c->trace_on && !c->g_full) CK(capture(c, &c->g_full, true, nullptr), "capture");
  const bool chunks = n >= 2 && prefill_eligible(c);
  if (chunks) CK(prefill_buffers(c), "prefill buffers");
  CK(cudaEventRecord(c->ev0, c->stream), "event");
  for (size_t i = 0; chunks && i < n; i += PF_CHUNK) {
    const int M = (int)std::min<size_t>(PF_CHUNK, n - i);
    CK(prefill_chunk(c, c->tokens_dev + i, M, c->pos + (uint32_t)i, false), "prefill");
    if (i + M == n) CK(enqueue_head(c), "head");
  }
  for (size_t i = 0; !chunks && i < n; ++i) {
    CK(cudaMemcpyAsync(c->token_dev, c->tokens_dev + i, 4, cudaMemcpyDeviceToDevice, c->stream), "token");
    const bool last = i + 1 == n;
    if (c->trace_on) {
      CK(enqueue_body(c, true), "forward");
      if (last) CK(enqueue_head(c), "head");
    } else {
      CK(cudaGraphLaunch(last ? c->g_full : c->g_body, c->stream), "graph launch");
    }
  }
  CK(cudaEventRecord(c->ev1, c->stream), "event");
  if (logits_out)
    CK(cudaMemcpyAsync(logits_out, c->logits, (size_t)mi.n_vocab * 4, cudaMemcpyDeviceToHost, c->stream),
       "logits copy");
  enqueue_err_read(c);
  CK(cudaStreamSynchronize(c->stream), "eval");
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, c->ev0, c->ev1);
  c->last_seconds = ms / 1e3;
  c->pos += (uint32_t)n;
  return check_err(c);
}

// The logits of every token of `tokens` (speculative verification of a
// draft, planned upstream in README.md:86-89; upstream's forward_batch keeps
// only the last row, src/forward.c:405-408). Ternary models take the chunk
// path (one tensor-core pass per projection) with the head on every row;
// others step. Each row equals the step-by-step logits of that token.
extern "C" foxcuda_status foxcuda_eval_all(foxcuda_context* c, const uint32_t* tokens, size_t n,
                                           float* logits_out) {
  if (!c || !tokens || n == 0 || !logits_out) return fail(FOXCUDA_ERR_ARG, "eval_all: nothing to evaluate");
  if (c->m->tp_size > 1)
    return fail(FOXCUDA_ERR_ARG, "eval_all: a tensor-parallel shard decodes through foxcuda_tp_*");
  const foxcuda_model_info& mi = c->m->info;
  const size_t nv = mi.n_vocab;
  if ((size_t)c->pos + n > c->n_ctx)
    return fail(FOXCUDA_ERR_ARG, "forward: %zu tokens past position %u would overrun the %u token context",
                n, c->pos, c->n_ctx);
  for (size_t i = 0; i < n; ++i)
    if (tokens[i] >= mi.n_vocab)
      return fail(FOXCUDA_ERR_ARG, "forward: token %u is outside the %u entry vocabulary", tokens[i], mi.n_vocab);
  cudaSetDevice(c->m->device);
  if (n > c->tokens_cap) {
    void* p = nullptr;
    CK(ctx_alloc(c, n * 4, &p), "token staging");
    c->tokens_dev = (uint32_t*)p;
    c->tokens_cap = n;
  }
  if (n > c->rows_cap) {
    void* p = nullptr;
    CK(ctx_alloc(c, n * nv * 4, &p), "logits staging");
    c->rows_logits = (float*)p;
    c->rows_cap = n;
  }
  CK(cudaMemcpyAsync(c->tokens_dev, tokens, n * 4, cudaMemcpyHostToDevice, c->stream), "token upload");
  const bool ternary = tc_layers_ok(c->m), kquant = !ternary && kq_layers_ok(c->m);
  const bool chunks = n >= 2 && !c->trace_on && (ternary || kquant);
  if (!chunks && !c->trace_on && !c->g_full) CK(capture(c, &c->g_full, true, nullptr), "capture");
  if (chunks) CK(prefill_buffers(c), "prefill buffers");
  CK(cudaEventRecord(c->ev0, c->stream), "event");
  for (size_t i = 0; chunks && i < n; i += PF_CHUNK) {
    const int M = (int)std::min<size_t>(PF_CHUNK, n - i);
    CK(kquant ? prefill_chunk_kq(c, c->tokens_dev + i, M, c->pos + (uint32_t)i, true)
              : prefill_chunk(c, c->tokens_dev + i, M, c->pos + (uint32_t)i, true),
       "prefill");
    if (kquant && is_kq(c->m->output.type)) {
      // a K-quant head quantises its input per 256 block like the layers:
      // one K-quant pass gives every row's logits (the decode head's values)
      const PackedMat& H = c->m->output;
      CK(quant_rows_k<true>(c, c->pf_x, (int)mi.n_embd, c->m->out_norm, decode_threads(H), M), "head rows");
      CK(kq_rows(c, H, M, c->rows_logits + i * nv, (int)nv), "head pass");
      continue;
    }
    for (int t = 0; t < M; ++t) {
      CK(cudaMemcpyAsync(c->x, c->pf_x + (size_t)t * mi.n_embd, (size_t)mi.n_embd * 4,
                         cudaMemcpyDeviceToDevice, c->stream), "row");
      CK(launch_head_on(c, c->stream, false), "head");
      CK(cudaMemcpyAsync(c->rows_logits + (i + t) * nv, c->logits, nv * 4, cudaMemcpyDeviceToDevice,
                         c->stream), "logits row");
    }
  }
  for (size_t i = 0; !chunks && i < n; ++i) {
    CK(cudaMemcpyAsync(c->token_dev, c->tokens_dev + i, 4, cudaMemcpyDeviceToDevice, c->stream), "token");
    if (c->trace_on) {
      CK(enqueue_body(c, true), "forward");
      CK(enqueue_head(c), "head");
    } else {
      CK(cudaGraphLaunch(c->g_full, c->stream), "graph launch");
    }
    CK(cudaMemcpyAsync(c->rows_logits + i * nv, c->logits, nv * 4, cudaMemcpyDeviceToDevice, c->stream),
       "logits row");
  }
  CK(cudaEventRecord(c->ev1, c->stream), "event");
  CK(cudaMemcpyAsync(logits_out, c->rows_logits, n * nv * 4, cudaMemcpyDeviceToHost, c->stream), "logits copy");
  enqueue_err_read(c);
  CK(cudaStreamSynchronize(c->stream), "eval_all");
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, c->ev0, c->ev1);
  c->last_seconds = ms / 1e3;
  c->pos += (uint32_t)n;
  return check_err(c);
}

// ---------------------------------------------------------------------------
// decode batches: one pass per step over several contexts of one model

constexpr int BATCH_MAX = 64;  // one token tile of the tensor-core pass

struct foxcuda_batch {
  foxcuda_model* m = nullptr;
  std::vector<foxcuda_context*> ctx;
  int n = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  double last_seconds = 0.0;
  // per sequence (device arrays): position, token, layer-0 K and V caches
  int** pos = nullptr;
  uint32_t** tokp = nullptr;
  void** kbase = nullptr;
  void** vbase = nullptr;
  const int** tables = nullptr;  // block tables of paged contexts (else nullptr)
  uint32_t* toks = nullptr;
  // rows of the pass, one per sequence
  float *x = nullptr, *xs = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr;
  float *gu = nullptr, *h = nullptr, *t = nullptr;
  int8_t* xq = nullptr;
  float* lg = nullptr;  // every sequence's logits (a K-quant head in one pass)
  std::vector<void*> allocs;
  cudaGraphExec_t graph = nullptr;  // a step and the picks, for foxcuda_batch_generate
  std::vector<foxcuda_sampler*> graph_samplers;
  std::vector<std::pair<cudaEvent_t, int>>* prof = nullptr;  // phase marks (foxcuda_batch_profile)
};

// An event after the launches of one phase of a profiled batch step.
static void bmark(foxcuda_batch* b, int kind) {
  if (!b->prof) return;
  cudaEvent_t e;
  if (cudaEventCreate(&e) != cudaSuccess) return;
  cudaEventRecord(e, b->stream);
  b->prof->push_back({e, kind});
}

extern "C" void foxcuda_batch_destroy(foxcuda_batch* b) {
  if (!b) return;
  cudaSetDevice(b->m->device);
  if (b->stream) cudaStreamSynchronize(b->stream);
  if (b->graph) cudaGraphExecDestroy(b->graph);
  for (void* p : b->allocs) cudaFree(p);
  if (b->ev0) cudaEventDestroy(b->ev0);
  if (b->ev1) cudaEventDestroy(b->ev1);
  if (b->stream) cudaStreamDestroy(b->stream);
  delete b;
}

extern "C" foxcuda_status foxcuda_batch_create(foxcuda_context* const* ctxs, size_t n, foxcuda_batch** out) {
  if (!ctxs || !out || n == 0) return fail(FOXCUDA_ERR_ARG, "batch: no contexts");
  *out = nullptr;
  if (n > (size_t)BATCH_MAX) return fail(FOXCUDA_ERR_ARG, "batch: %zu contexts; at most %d", n, BATCH_MAX);
  foxcuda_context* c0 = ctxs[0];
  for (size_t i = 0; i < n; ++i) {
    const foxcuda_context* c = ctxs[i];
    if (!c) return fail(FOXCUDA_ERR_ARG, "batch: context %zu is null", i);
    if (c->m != c0->m) return fail(FOXCUDA_ERR_ARG, "batch: the contexts use different models");
    if (c->n_ctx != c0->n_ctx || c->kv_f16 != c0->kv_f16 || c->attn_exact != c0->attn_exact)
      return fail(FOXCUDA_ERR_ARG, "batch: the contexts differ in length, cache type or attention mode");
    if (c->pool != c0->pool)
      return fail(FOXCUDA_ERR_ARG, "batch: the contexts' caches are not all from the same page pool "
                  "(or all contiguous)");
    for (size_t j = 0; j < i; ++j)
      if (ctxs[j] == c) return fail(FOXCUDA_ERR_ARG, "batch: context %zu appears twice", i);
  }
  foxcuda_model* m = c0->m;
  if (!tc_layers_ok(m))
    return fail(FOXCUDA_ERR_UNSUPPORTED, "batch: the batched step needs single-GPU ternary layer "
                "matrices (held as TQ2_0)");
  cudaSetDevice(m->device);
  foxcuda_batch* b = new foxcuda_batch();
  b->m = m;
  b->ctx.assign(ctxs, ctxs + n);
  b->n = (int)n;
  const foxcuda_model_info& mi = m->info;
  const size_t E = mi.n_embd, nq = (size_t)mi.n_head * mi.head_dim, nkv = (size_t)mi.n_head_kv * mi.head_dim;
  const size_t F = mi.n_ff, kmax = std::max(E, std::max(nq, F));
  cudaError_t e = cudaSuccess;
  auto A = [&](size_t bytes, void** p) {
    if (e != cudaSuccess) return;
    e = cudaMalloc(p, bytes ? bytes : 16);
    if (e == cudaSuccess) b->allocs.push_back(*p);
  };
  A(n * sizeof(int*), (void**)&b->pos);
  A(n * sizeof(uint32_t*), (void**)&b->tokp);
  A(n * sizeof(void*), (void**)&b->kbase);
  A(n * sizeof(void*), (void**)&b->vbase);
  A(n * 4, (void**)&b->toks);
  A(n * E * 4, (void**)&b->x);
  A(n * kmax, (void**)&b->xq);
  A(n * (kmax / 256 + 1) * 4, (void**)&b->xs);  // per token, or per 256 block (a K-quant head)
  if (is_kq(m->output.type)) A(n * (size_t)mi.n_vocab * 4, (void**)&b->lg);
  A(n * (nq + 2 * nkv) * 4, (void**)&b->qkv);
  A(n * nq * 4, (void**)&b->q);
  A(n * nq * 4, (void**)&b->att);
  A(n * 2 * F * 4, (void**)&b->gu);
  A(n * F * 4, (void**)&b->h);
  A(n * E * 4, (void**)&b->t);
  std::vector<int*> pos(n);
  std::vector<uint32_t*> tokp(n);
  std::vector<void*> kb(n), vb(n);
  for (size_t i = 0; i < n; ++i) {
    pos[i] = ctxs[i]->pos_dev; tokp[i] = ctxs[i]->token_dev; kb[i] = ctxs[i]->kc; vb[i] = ctxs[i]->vc;
  }
  if (e == cudaSuccess) e = cudaMemcpy(b->pos, pos.data(), n * sizeof(int*), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(b->tokp, tokp.data(), n * sizeof(uint32_t*), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(b->kbase, kb.data(), n * sizeof(void*), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(b->vbase, vb.data(), n * sizeof(void*), cudaMemcpyHostToDevice);
  if (c0->pool) {
    std::vector<const int*> tb(n);
    for (size_t i = 0; i < n; ++i) tb[i] = ctxs[i]->kv_table;
    A(n * sizeof(int*), (void**)&b->tables);
    if (e == cudaSuccess) e = cudaMemcpy(b->tables, tb.data(), n * sizeof(int*), cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreate(&b->ev0);
  if (e == cudaSuccess) e = cudaEventCreate(&b->ev1);
  if (e != cudaSuccess) {
    foxcuda_batch_destroy(b);
    return cuda_fail(e, "batch allocation");
  }
  *out = b;
  return FOXCUDA_OK;
}

// One token of every sequence through the layers and the head. Row i is
// sequence i: its token (gathered from its context, or already in b->toks),
// its position, its caches. Per sequence the values are its decode step's:
// the tensor-core pass gives each row its single-token GEMV, and every other
// kernel is the decode step's or repeats its arithmetic row-wise.
static cudaError_t enqueue_batch_body(foxcuda_batch* b, bool gather) {
  foxcuda_model* m = b->m;
  const foxcuda_model_info& mi = m->info;
  cudaStream_t s = b->stream;
  foxcuda_context* c0 = b->ctx[0];
  const int M = b->n, E = mi.n_embd, hd = mi.head_dim;
  const int nq = mi.n_head * hd, nkv = mi.n_head_kv * hd, F = mi.n_ff, nqkv = nq + 2 * nkv;
  const float eps = mi.rms_eps;
  const size_t layer_bytes = c0->kv_layer_elems * (c0->kv_f16 ? 2 : 4);
  const size_t rows_e = (size_t)M * E;
  const unsigned add_grid = (unsigned)std::min<size_t>((rows_e + 255) / 256, 4096);
  if (gather) gather_tokens_kernel<<<1, BATCH_MAX, 0, s>>>(b->tokp, M, b->toks);
  embed_rows_kernel<<<dim3((E + 255) / 256, M), 256, 0, s>>>(m->embd.type, m->embd.dev,
                                                            row_bytes(m->embd.type, E), E, b->toks, b->x);
  cudaError_t e = cudaGetLastError();
  bmark(b, PK_EMBED);
  for (uint32_t l = 0; l < mi.n_layer && !e; ++l) {
    const LayerW& L = m->layers[l];
    if ((e = quant_rows_to<true>(b->x, E, L.attn_norm, eps, decode_threads(L.qkv[0]), M, b->xq, b->xs, s)))
      break;
    if ((e = tc_rows_to(b->xq, b->xs, L.qkv[0], M, b->qkv, c0->err_dev, s))) break;
    qkv_seqs_kernel<<<dim3((nqkv + 255) / 256, M), 256, 0, s>>>(
        b->qkv, nqkv, nq, nkv, hd, (int)c0->n_ctx, b->pos, b->kbase, b->vbase, (size_t)l * layer_bytes,
        b->tables, c0->rope_cos, c0->rope_sin, c0->kv_f16, b->q);
    if ((e = cudaGetLastError())) break;
    bmark(b, PK_QKV);
    AttnParams all{};
    all.q = b->q; all.out = b->att; all.seq_stride = nq;
    all.pos_list = b->pos; all.k_list = b->kbase; all.v_list = b->vbase; all.layer_off = (size_t)l * layer_bytes;
    all.table_list = b->tables;
    all.kv_f16 = c0->kv_f16; all.n_ctx = c0->n_ctx;
    all.hd = hd; all.n_head = mi.n_head; all.n_kv = mi.n_head_kv; all.nt = m->attn_nt;
    all.scale = 1.0f / sqrtf((float)hd);
    if (!c0->attn_exact) {
      e = launch_tiles(all, M, s);
    } else {
      for (int i = 0; i < M && !e; ++i) {
        foxcuda_context* c = b->ctx[i];
        AttnParams ap{};
        ap.q = b->q + (size_t)i * nq; ap.kcache = kv_layer(c, c->kc, l); ap.vcache = kv_layer(c, c->vc, l);
        ap.kv_table = c->kv_table;
        ap.kv_f16 = c->kv_f16; ap.n_ctx = c->n_ctx;
        ap.hd = hd; ap.n_head = mi.n_head; ap.n_kv = mi.n_head_kv; ap.nt = m->attn_nt;
        ap.pos = c->pos_dev; ap.out = b->att + (size_t)i * nq;
        ap.scale = 1.0f / sqrtf((float)hd);
        e = run_attention(ap, c->attn_exact, s);
      }
    }
    if (e) break;
    bmark(b, PK_ATTN);
    if ((e = quant_rows_to<false>(b->att, nq, nullptr, eps, 256, M, b->xq, b->xs, s))) break;
    if ((e = tc_rows_to(b->xq, b->xs, L.o, M, b->t, c0->err_dev, s))) break;
    add_rows_kernel<<<add_grid, 256, 0, s>>>(b->x, b->t, rows_e);
    bmark(b, PK_O);
    if ((e = quant_rows_to<true>(b->x, E, L.ffn_norm, eps, decode_threads(L.gateup), M, b->xq, b->xs, s)))
      break;
    if ((e = tc_rows_to(b->xq, b->xs, L.gateup, M, b->gu, c0->err_dev, s))) break;
    swiglu_rows_kernel<<<dim3((F + 255) / 256, M), 256, 0, s>>>(b->gu, 2 * F, L.gateup.U, b->h);
    bmark(b, PK_GATEUP);
    if ((e = quant_rows_to<false>(b->h, F, nullptr, eps, 256, M, b->xq, b->xs, s))) break;
    if ((e = tc_rows_to(b->xq, b->xs, L.down, M, b->t, c0->err_dev, s))) break;
    add_rows_kernel<<<add_grid, 256, 0, s>>>(b->x, b->t, rows_e);
    e = cudaGetLastError();
    bmark(b, PK_DOWN);
  }
  if (!e && b->lg) {
    // a K-quant head quantises per 256 block like the layers: one K-quant
    // pass gives every sequence's logits (each its decode head's values)
    const PackedMat& H = m->output;
    const size_t nv = mi.n_vocab;
    e = quant_rows_k_to<true>(b->x, E, m->out_norm, eps, decode_threads(H), M, b->xq, b->xs, s);
    if (!e) e = kq_rows_to(b->xq, b->xs, H, M, b->lg, (int)nv, c0->err_dev, s);
    for (int i = 0; i < M && !e; ++i)
      e = cudaMemcpyAsync(b->ctx[i]->logits, b->lg + i * nv, nv * 4, cudaMemcpyDeviceToDevice, s);
  } else {
    // each sequence's head on its own residual row, into its context's logits
    for (int i = 0; i < M && !e; ++i) {
      foxcuda_context* c = b->ctx[i];
      e = cudaMemcpyAsync(c->x, b->x + (size_t)i * E, (size_t)E * 4, cudaMemcpyDeviceToDevice, s);
      if (!e) e = launch_head_on(c, s, false);
    }
  }
  if (e) return e;
  bmark(b, PK_HEAD);
  advance_all_kernel<<<1, BATCH_MAX, 0, s>>>(b->pos, M);
  bmark(b, PK_ADVANCE);
  return cudaGetLastError();
}

static foxcuda_status batch_begin(foxcuda_batch* b, size_t steps) {
  for (foxcuda_context* c : b->ctx)
    if ((size_t)c->pos + steps > c->n_ctx)
      return fail(FOXCUDA_ERR_ARG, "batch: %zu tokens past position %u would overrun the %u token context",
                  steps, c->pos, c->n_ctx);
  cudaSetDevice(b->m->device);
  for (foxcuda_context* c : b->ctx) CK(cudaStreamSynchronize(c->stream), "batch: context stream");
  return FOXCUDA_OK;
}

// The device error word of every context (bounded waits that gave up).
static foxcuda_status batch_errors(foxcuda_batch* b) {
  for (foxcuda_context* c : b->ctx) {
    uint32_t code = 0;
    CK(cudaMemcpy(&code, c->err_dev, 4, cudaMemcpyDeviceToHost), "batch: error word");
    if (code) {
      cudaMemset(c->err_dev, 0, 4);
      return fail(FOXCUDA_ERR_INTERNAL, "device: a bounded wait gave up (code %u); the step's outputs "
                  "are not valid", code);
    }
  }
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_batch_step(foxcuda_batch* b, const uint32_t* tokens, float* logits) {
  if (!b) return fail(FOXCUDA_ERR_ARG, "batch: null batch");
  const uint32_t nv = b->m->info.n_vocab;
  if (tokens)
    for (int i = 0; i < b->n; ++i)
      if (tokens[i] >= nv) return fail(FOXCUDA_ERR_ARG, "forward: token %u is outside the vocabulary", tokens[i]);
  foxcuda_status st = batch_begin(b, 1);
  if (st) return st;
  if (tokens) CK(cudaMemcpyAsync(b->toks, tokens, (size_t)b->n * 4, cudaMemcpyHostToDevice, b->stream), "tokens");
  CK(cudaEventRecord(b->ev0, b->stream), "event");
  CK(enqueue_batch_body(b, tokens == nullptr), "batch step");
  CK(cudaEventRecord(b->ev1, b->stream), "event");
  for (int i = 0; logits && i < b->n; ++i)
    CK(cudaMemcpyAsync(logits + (size_t)i * nv, b->ctx[i]->logits, (size_t)nv * 4, cudaMemcpyDeviceToHost,
                       b->stream), "logits copy");
  CK(cudaStreamSynchronize(b->stream), "batch step");
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, b->ev0, b->ev1);
  b->last_seconds = ms / 1e3;
  for (foxcuda_context* c : b->ctx) c->pos += 1;
  return batch_errors(b);
}

// One batch step (as foxcuda_batch_step, no logits copied out) with an
// event after each phase: kinds and microseconds per phase, as
// foxcuda_context_profile gives them for a decode step.
extern "C" foxcuda_status foxcuda_batch_profile(foxcuda_batch* b, const uint32_t* tokens, float* us,
                                                int* kinds, int cap, int* n_out) {
  if (!b || !tokens || !us || !kinds || !n_out || cap <= 0) return fail(FOXCUDA_ERR_ARG, "batch profile: bad argument");
  const uint32_t nv = b->m->info.n_vocab;
  for (int i = 0; i < b->n; ++i)
    if (tokens[i] >= nv) return fail(FOXCUDA_ERR_ARG, "forward: token %u is outside the vocabulary", tokens[i]);
  foxcuda_status st = batch_begin(b, 1);
  if (st) return st;
  CK(cudaMemcpyAsync(b->toks, tokens, (size_t)b->n * 4, cudaMemcpyHostToDevice, b->stream), "tokens");
  std::vector<std::pair<cudaEvent_t, int>> marks;
  CK(cudaEventRecord(b->ev0, b->stream), "event");
  b->prof = &marks;
  cudaError_t e = enqueue_batch_body(b, false);
  b->prof = nullptr;
  cudaError_t e2 = cudaStreamSynchronize(b->stream);
  int n = 0;
  cudaEvent_t prev = b->ev0;
  for (auto& mk : marks) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, prev, mk.first);
    if (n < cap) { us[n] = ms * 1e3f; kinds[n] = mk.second; ++n; }
    if (prev != b->ev0) cudaEventDestroy(prev);
    prev = mk.first;
  }
  if (prev != b->ev0) cudaEventDestroy(prev);
  *n_out = n;
  if (e) return cuda_fail(e, "batch profile");
  CK(e2, "batch profile");
  for (foxcuda_context* c : b->ctx) c->pos += 1;
  return batch_errors(b);
}

extern "C" foxcuda_status foxcuda_batch_generate(foxcuda_batch* b, foxcuda_sampler* const* samplers,
                                                 const uint32_t* first, size_t n_steps, uint32_t* out) {
  if (!b || !samplers || !out || n_steps == 0) return fail(FOXCUDA_ERR_ARG, "batch: nothing to generate");
  const uint32_t nv = b->m->info.n_vocab;
  for (int i = 0; i < b->n; ++i) {
    if (!samplers[i] || samplers[i]->c != b->ctx[i])
      return fail(FOXCUDA_ERR_ARG, "batch: sampler %d does not belong to context %d", i, i);
    if (first && first[i] >= nv) return fail(FOXCUDA_ERR_ARG, "forward: token %u is outside the vocabulary", first[i]);
  }
  foxcuda_status st = batch_begin(b, n_steps);
  if (st) return st;
  const bool same = b->graph && std::equal(b->graph_samplers.begin(), b->graph_samplers.end(), samplers);
  if (!same) {
    if (b->graph) cudaGraphExecDestroy(b->graph);
    b->graph = nullptr;
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal), "capture");
    cudaError_t e = enqueue_batch_body(b, true);
    for (int i = 0; i < b->n && !e; ++i) e = enqueue_pick_on(samplers[i], true, b->stream);
    cudaError_t e2 = cudaStreamEndCapture(b->stream, &g);
    if (e || e2) {
      if (g) cudaGraphDestroy(g);
      return cuda_fail(e ? e : e2, "batch capture");
    }
    e = cudaGraphInstantiate(&b->graph, g, 0);
    cudaGraphDestroy(g);
    CK(e, "batch graph");
    b->graph_samplers.assign(samplers, samplers + b->n);
  }
  if (first)
    for (int i = 0; i < b->n; ++i)
      CK(cudaMemcpyAsync(b->ctx[i]->token_dev, first + i, 4, cudaMemcpyHostToDevice, b->stream), "token in");
  std::vector<uint32_t> start(b->n);
  for (int i = 0; i < b->n; ++i) start[i] = samplers[i]->n_out;
  CK(cudaEventRecord(b->ev0, b->stream), "event");
  for (size_t k = 0; k < n_steps; ++k) CK(cudaGraphLaunch(b->graph, b->stream), "graph launch");
  CK(cudaEventRecord(b->ev1, b->stream), "event");
  CK(cudaStreamSynchronize(b->stream), "batch generate");
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, b->ev0, b->ev1);
  b->last_seconds = ms / 1e3;
  std::vector<uint32_t> picks(n_steps);
  for (int i = 0; i < b->n; ++i) {
    foxcuda_context* c = b->ctx[i];
    samplers[i]->n_out += (uint32_t)n_steps;
    c->pos += (uint32_t)n_steps;
    const uint32_t cap = c->n_ctx;
    for (size_t k = 0; k < n_steps;) {  // the ring may wrap
      const uint32_t at = (start[i] + (uint32_t)k) % cap;
      const size_t run = std::min<size_t>(n_steps - k, cap - at);
      CK(cudaMemcpy(picks.data() + k, c->ring + at, run * 4, cudaMemcpyDeviceToHost), "ring copy");
      k += run;
    }
    for (size_t k = 0; k < n_steps; ++k) out[k * b->n + i] = picks[k];
  }
  return batch_errors(b);
}

extern "C" double foxcuda_batch_last_seconds(const foxcuda_batch* b) { return b ? b->last_seconds : 0.0; }

extern "C" foxcuda_status foxcuda_context_fill_kv(foxcuda_context* c, uint32_t n_pos, uint64_t seed) {
  if (!c) return fail(FOXCUDA_ERR_ARG, "fill_kv: null context");
  if (n_pos > c->n_ctx) return fail(FOXCUDA_ERR_ARG, "fill_kv: %u positions in a %u token context", n_pos, c->n_ctx);
  const foxcuda_model_info& mi = c->m->loc;
  cudaSetDevice(c->m->device);
  CK(cudaStreamSynchronize(c->stream), "fill_kv");
  const size_t runs = (size_t)mi.n_layer * mi.n_head_kv;
  const size_t total = runs * n_pos * mi.head_dim;
  const unsigned grid = (unsigned)std::max<size_t>(1, std::min<size_t>((total + 255) / 256, 16384));
  if (total) {
    fill_kv_kernel<<<grid, 256, 0, c->stream>>>(c->kc, c->kv_f16, runs, (int)c->n_ctx, (int)mi.head_dim,
                                                (int)n_pos, (int)mi.n_head_kv, c->kv_layer_elems, c->kv_table,
                                                seed);
    fill_kv_kernel<<<grid, 256, 0, c->stream>>>(c->vc, c->kv_f16, runs, (int)c->n_ctx, (int)mi.head_dim,
                                                (int)n_pos, (int)mi.n_head_kv, c->kv_layer_elems, c->kv_table,
                                                ~seed);
    CK(cudaGetLastError(), "fill_kv launch");
  }
  const int p = (int)n_pos;
  CK(cudaMemcpyAsync(c->pos_dev, &p, 4, cudaMemcpyHostToDevice, c->stream), "position");
  CK(cudaStreamSynchronize(c->stream), "fill_kv");
  c->pos = n_pos;
  return FOXCUDA_OK;
}

// ---------------------------------------------------------------------------
// sampler

extern "C" foxcuda_status foxcuda_sampler_create(foxcuda_context* c, const foxcuda_sampler_config* cfg,
                                                 foxcuda_sampler** out) {
  if (!c || !out) return fail(FOXCUDA_ERR_ARG, "sampler: null argument");
  *out = nullptr;
  if (c->m->tp_size > 1)
    return fail(FOXCUDA_ERR_ARG, "sampler: a tensor-parallel shard picks through foxcuda_tp_*");
  foxcuda_sampler_config k;
  if (cfg) k = *cfg;
  else k = {0.8f, 40, 0.95f, 1.1f, 64, 0};  // upstream defaults, src/sample.c:21-30
  // upstream src/sample.c:59-66
  if (k.top_k < 0) k.top_k = 0;
  if (k.top_k > TOPK_MAX) k.top_k = TOPK_MAX;
  if (k.top_p <= 0.0f || k.top_p > 1.0f) k.top_p = 1.0f;
  if (k.repeat_penalty < 1.0f) k.repeat_penalty = 1.0f;
  if (k.repeat_last_n > SAMPLER_MAX_HIST)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "sampler: repeat_last_n %u is above %d", k.repeat_last_n, SAMPLER_MAX_HIST);
  cudaSetDevice(c->m->device);
  foxcuda_sampler* s = new foxcuda_sampler();
  s->c = c;
  s->cfg = k;
  const int nv = (int)c->m->info.n_vocab;
  s->k = (k.top_k <= 0 || k.top_k > nv) ? std::min(nv, TOPK_MAX) : k.top_k;
  cudaError_t e = cudaMalloc(&s->dev, sizeof(SamplerDev));
  if (e == cudaSuccess) e = cudaMemset(s->dev, 0, sizeof(SamplerDev));
  if (e == cudaSuccess) {
    const uint32_t cap = k.repeat_last_n ? k.repeat_last_n : 1;
    const unsigned long long rng = k.seed ? k.seed : 0x9E3779B97F4A7C15ull;
    e = cudaMemcpy(&s->dev->hist_cap, &cap, 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(&s->dev->rng, &rng, 8, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) {
    if (s->dev) cudaFree(s->dev);
    delete s;
    return cuda_fail(e, "sampler alloc");
  }
  *out = s;
  return FOXCUDA_OK;
}

extern "C" void foxcuda_sampler_destroy(foxcuda_sampler* s) {
  if (!s) return;
  cudaSetDevice(s->c->m->device);
  cudaStreamSynchronize(s->c->stream);
  if (s->g_decode) cudaGraphExecDestroy(s->g_decode);
  cudaFree(s->dev);
  delete s;
}

extern "C" foxcuda_status foxcuda_sampler_accept(foxcuda_sampler* s, uint32_t token) {
  if (!s) return fail(FOXCUDA_ERR_ARG, "sampler: null");
  cudaSetDevice(s->c->m->device);
  accept_kernel<<<1, 32, 0, s->c->stream>>>(s->dev, token);
  CK(cudaGetLastError(), "accept");
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_sampler_pick(foxcuda_sampler* s, uint32_t* out) {
  if (!s || !out) return fail(FOXCUDA_ERR_ARG, "sampler: null argument");
  foxcuda_context* c = s->c;
  cudaSetDevice(c->m->device);
  CK(enqueue_pick(s, false), "pick");
  s->n_out++;
  CK(cudaMemcpyAsync(c->h_pinned + 1, c->token_dev, 4, cudaMemcpyDeviceToHost, c->stream), "pick copy");
  CK(cudaStreamSynchronize(c->stream), "pick");
  *out = c->h_pinned[1];
  return FOXCUDA_OK;
}

static foxcuda_status decode_steps(foxcuda_context* c, foxcuda_sampler* s, uint32_t token, size_t n,
                                   uint32_t* out) {
  const foxcuda_model_info& mi = c->m->info;
  if (token >= mi.n_vocab) return fail(FOXCUDA_ERR_ARG, "forward: token %u is outside the vocabulary", token);
  if ((size_t)c->pos + n > c->n_ctx)
    return fail(FOXCUDA_ERR_ARG, "forward: %zu tokens past position %u would overrun the %u token context",
                n, c->pos, c->n_ctx);
  cudaSetDevice(c->m->device);
  if (!s->g_decode) CK(capture(c, &s->g_decode, true, s), "capture");
  c->h_pinned[0] = token;
  CK(cudaMemcpyAsync(c->token_dev, c->h_pinned, 4, cudaMemcpyHostToDevice, c->stream), "token in");
  CK(cudaEventRecord(c->ev0, c->stream), "event");
  const uint32_t start = s->n_out;
  for (size_t i = 0; i < n; ++i) CK(cudaGraphLaunch(s->g_decode, c->stream), "graph launch");
  CK(cudaEventRecord(c->ev1, c->stream), "event");
  s->n_out += (uint32_t)n;
  if (n == 1) {
    // the picked token and the device error code in one 8-byte copy
    CK(cudaMemcpyAsync(c->h_pinned + 1, c->token_dev, 8, cudaMemcpyDeviceToHost, c->stream), "token out");
    CK(cudaStreamSynchronize(c->stream), "decode");
    out[0] = c->h_pinned[1];
    c->h_pinned[3] = c->h_pinned[2];
  } else {
    enqueue_err_read(c);
    CK(cudaStreamSynchronize(c->stream), "generate");
    const uint32_t cap = c->n_ctx;
    for (size_t i = 0; i < n;) {  // the ring may wrap
      const uint32_t at = (start + (uint32_t)i) % cap;
      const size_t run = std::min<size_t>(n - i, cap - at);
      CK(cudaMemcpy(out + i, c->ring + at, run * 4, cudaMemcpyDeviceToHost), "ring copy");
      i += run;
    }
  }
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, c->ev0, c->ev1);
  c->last_seconds = ms / 1e3;
  c->pos += (uint32_t)n;
  return check_err(c);
}

extern "C" foxcuda_status foxcuda_decode(foxcuda_context* c, foxcuda_sampler* s, uint32_t token,
                                         uint32_t* next) {
  if (!c || !s || !next || s->c != c) return fail(FOXCUDA_ERR_ARG, "decode: bad argument");
  return decode_steps(c, s, token, 1, next);
}

extern "C" foxcuda_status foxcuda_generate(foxcuda_context* c, foxcuda_sampler* s, uint32_t token,
                                           size_t n, uint32_t* out) {
  if (!c || !s || !out || s->c != c || n == 0) return fail(FOXCUDA_ERR_ARG, "generate: bad argument");
  return decode_steps(c, s, token, n, out);
}

// ---------------------------------------------------------------------------
// tensor-parallel decode steps (stream-ordered on the context's stream; the
// caller puts its collectives on the same stream between them)

extern "C" void* foxcuda_context_stream(foxcuda_context* c) { return c ? (void*)c->stream : nullptr; }

extern "C" foxcuda_status foxcuda_tp_info(const foxcuda_model* m, foxcuda_tp_shape* out) {
  if (!m || !out) return fail(FOXCUDA_ERR_ARG, "tp_info: null argument");
  out->tp_rank = m->tp_rank;
  out->tp_size = m->tp_size;
  out->n_head = m->loc.n_head;
  out->n_head_kv = m->loc.n_head_kv;
  out->n_ff = m->loc.n_ff;
  out->vocab_begin = m->vocab0;
  out->n_vocab = m->loc.n_vocab;
  out->o_blocks = m->o_blocks;
  for (int k = 0; k < 8; ++k) out->ffn_blocks[k] = m->f_blocks_all[k];
  auto nt = [](int t) -> uint32_t { return t == T_Q4_K ? 8 : t == T_Q6_K ? 4 : 1; };
  out->o_terms = out->down_terms = 1;
  if (m->finalized)
    for (const LayerW& L : m->layers) {
      out->o_terms = std::max(out->o_terms, nt(L.o.type));
      out->down_terms = std::max(out->down_terms, nt(L.down.type));
    }
  return FOXCUDA_OK;
}

static foxcuda_status tp_check(foxcuda_context* c, uint32_t layer, bool need_layer) {
  if (!c) return fail(FOXCUDA_ERR_ARG, "tp: null context");
  if (need_layer && layer >= c->m->info.n_layer) return fail(FOXCUDA_ERR_ARG, "tp: layer %u", layer);
  if (c->pos >= c->n_ctx) return fail(FOXCUDA_ERR_ARG, "tp: the %u token context is full", c->n_ctx);
  cudaSetDevice(c->m->device);
  c->tp_steps = true;
  return FOXCUDA_OK;
}

// Embedding of the token in device memory (set by foxcuda_tp_pick, or from
// the host with token < n_vocab).
extern "C" foxcuda_status foxcuda_tp_embed(foxcuda_context* c, int64_t token) {
  foxcuda_status st = tp_check(c, 0, false);
  if (st) return st;
  // A pending sums exchange is completed even though the embedding replaces
  // the residual: the completion waits for every rank's rows, and that wait
  // is what keeps any rank from pushing the next rows of the same kind into
  // an area another rank has not read yet (K-quant shards trade no absmax
  // that would order it otherwise).
  if ((st = flush_fold(c))) return st;
  const foxcuda_model_info& mi = c->m->info;
  const size_t emb_rb = row_bytes(c->m->embd.type, mi.n_embd);
  if (token >= 0) {
    // the token travels as a launch argument: these calls do not wait for
    // the device, so a staging word in host memory could be overwritten by
    // the next call before its copy ran
    if ((uint64_t)token >= mi.n_vocab) return fail(FOXCUDA_ERR_ARG, "tp: token outside the vocabulary");
    embed_token_kernel<<<(mi.n_embd + 255) / 256, 256, 0, c->stream>>>(
        c->m->embd.type, c->m->embd.dev, emb_rb, (int)mi.n_embd, (uint32_t)token, c->token_dev, c->x);
    // a host token (the prompt) enters the penalty history, as `fox run`
    // accepts the prompt into its sampler (src/cli.c:340-345)
    if (c->tp_smp) accept_kernel<<<1, 32, 0, c->stream>>>(c->tp_smp, (uint32_t)token);
  } else {
    embed_kernel<<<(mi.n_embd + 255) / 256, 256, 0, c->stream>>>(c->m->embd.type, c->m->embd.dev, emb_rb,
                                                                  (int)mi.n_embd, c->token_dev, c->x);
  }
  CK(cudaGetLastError(), "embed");
  if (c->trace_on)
    CK(cudaMemcpyAsync(c->trace, c->x, mi.n_embd * 4, cudaMemcpyDeviceToDevice, c->stream), "trace");
  return FOXCUDA_OK;
}

// q|k|v rows and attention of this shard's heads
extern "C" foxcuda_status foxcuda_tp_attention(foxcuda_context* c, uint32_t layer) {
  foxcuda_status st = tp_check(c, layer, true);
  if (st) return st;
  CK(launch_qkv(c, layer), "tp qkv");
  CK(launch_attn(c, layer), "tp attention");
  return FOXCUDA_OK;
}

// which: 0 = the attention output (o projection input), 1 = the FFN hidden
// vector (down projection input)
extern "C" foxcuda_status foxcuda_tp_amax(foxcuda_context* c, int which, float* amax) {
  foxcuda_status st = tp_check(c, 0, false);
  if (st) return st;
  if ((st = flush_fold(c))) return st;
  if (!amax || (which != 0 && which != 1)) return fail(FOXCUDA_ERR_ARG, "tp_amax: bad argument");
  const int n = which == 0 ? (int)(c->m->loc.n_head * c->m->info.head_dim) : (int)c->m->loc.n_ff;
  amax_kernel<<<1, 1024, 0, c->stream>>>(which == 0 ? c->att : c->h, n, amax);
  CK(cudaGetLastError(), "tp amax");
  return FOXCUDA_OK;
}

template <int T>
static cudaError_t launch_terms_t(const GemvParams& p, bool gscale, cudaStream_t s) {
  if (gscale) return launch_gemv_t<T, PRO_GSCALE, EPI_TERMS>(p, s);
  return launch_gemv_t<T, PRO_VEC, EPI_TERMS>(p, s);
}

// This shard's block terms of the o (which 0) or down (which 1) projection:
// terms[row * stride + j] for its column blocks. Ternary shards quantise with
// amax_all, the absmax over all shards; K-quant shards use their own 256-block
// scales, which are the unsplit vector's.
extern "C" foxcuda_status foxcuda_tp_terms(foxcuda_context* c, uint32_t layer, int which,
                                           const float* amax_all, float* terms, uint32_t stride) {
  foxcuda_status st = tp_check(c, layer, true);
  if (st) return st;
  if (!terms || (which != 0 && which != 1)) return fail(FOXCUDA_ERR_ARG, "tp_terms: bad argument");
  if ((st = flush_fold(c))) return st;
  const PackedMat& W = which == 0 ? c->m->layers[layer].o : c->m->layers[layer].down;
  const int nt = W.type == T_Q4_K ? 8 : W.type == T_Q6_K ? 4 : 1;
  if (stride < (uint32_t)(W.nb * nt)) return fail(FOXCUDA_ERR_ARG, "tp_terms: stride %u below %d", stride, W.nb * nt);
  const bool tern = W.type == T_TQ1_0 || W.type == T_TQ2_0;
  if (tern && !amax_all) return fail(FOXCUDA_ERR_ARG, "tp_terms: ternary shards need the global absmax");
  GemvParams p = gemv_base(W.type, W.dev, W.n_rows, W.K, W.nb, W.U);
  p.x = which == 0 ? c->att : c->h;
  p.xq_scale = amax_all;
  p.out = terms;
  p.terms_stride = (int)stride;
  p.err = c->err_dev;
  cudaError_t e;
  if (W.slice || W.stream) {
    CK(launch_sliced(W, PRO_GSCALE, EPI_TERMS, p, c->stream), "tp terms");
    return FOXCUDA_OK;
  }
  switch (W.type) {
    case T_TQ1_0: e = launch_terms_t<T_TQ1_0>(p, true, c->stream); break;
    case T_TQ2_0: e = launch_terms_t<T_TQ2_0>(p, true, c->stream); break;
    case T_Q4_K: e = launch_terms_t<T_Q4_K>(p, false, c->stream); break;
    case T_Q6_K: e = launch_terms_t<T_Q6_K>(p, false, c->stream); break;
    default: return fail(FOXCUDA_ERR_UNSUPPORTED, "tp_terms: type %d", W.type);
  }
  CK(e, "tp terms");
  return FOXCUDA_OK;
}

// Fold the gathered terms ([tp][n_embd][stride], shard order) into the
// residual stream.
extern "C" foxcuda_status foxcuda_tp_fold(foxcuda_context* c, uint32_t layer, int which,
                                          const float* gathered, uint32_t stride,
                                          const float* amax_all) {
  foxcuda_status st = tp_check(c, layer, true);
  if (st) return st;
  if (!gathered || (which != 0 && which != 1)) return fail(FOXCUDA_ERR_ARG, "tp_fold: bad argument");
  if ((st = flush_fold(c))) return st;
  const foxcuda_model* m = c->m;
  const PackedMat& W = which == 0 ? m->layers[layer].o : m->layers[layer].down;
  const int nt = W.type == T_Q4_K ? 8 : W.type == T_Q6_K ? 4 : 1;
  FoldParams f;
  memset(&f, 0, sizeof f);
  f.g = gathered;
  f.tp = m->tp_size;
  f.rows = (int)m->info.n_embd;
  f.stride = (int)stride;
  f.ternary = W.type == T_TQ1_0 || W.type == T_TQ2_0;
  for (int k = 0; k < m->tp_size; ++k) {
    const int blocks = which == 0 ? (int)m->o_blocks : (int)m->f_blocks_all[k];
    f.count[k] = blocks * nt;
    if ((uint32_t)f.count[k] > stride) return fail(FOXCUDA_ERR_ARG, "tp_fold: stride %u below %d", stride, f.count[k]);
  }
  f.amax = amax_all;
  f.x = c->x;
  if (f.ternary && !amax_all) return fail(FOXCUDA_ERR_ARG, "tp_fold: ternary shards need the global absmax");
  fold_kernel<<<(f.rows + 255) / 256, 256, 0, c->stream>>>(f);
  CK(cudaGetLastError(), "tp fold");
  if (c->trace_on && which == 1)  // the layer's output, as foxcuda_context_hidden reads it
    CK(cudaMemcpyAsync(c->trace + (size_t)(layer + 1) * m->info.n_embd, c->x, m->info.n_embd * 4,
                       cudaMemcpyDeviceToDevice, c->stream), "trace");
  return FOXCUDA_OK;
}

// gate|up rows of this shard's FFN blocks, SwiGLU into the hidden vector
extern "C" foxcuda_status foxcuda_tp_ffn(foxcuda_context* c, uint32_t layer) {
  foxcuda_status st = tp_check(c, layer, true);
  if (st) return st;
  CK(launch_gateup(c, layer), "tp gate|up");
  return FOXCUDA_OK;
}

// Head rows of this shard and their best logit as {value, global index bits}.
extern "C" foxcuda_status foxcuda_tp_head(foxcuda_context* c, float* best) {
  foxcuda_status st = tp_check(c, 0, false);
  if (st) return st;
  if (!best) return fail(FOXCUDA_ERR_ARG, "tp_head: null output");
  if ((st = flush_fold(c))) return st;
  CK(launch_head(c), "tp head");
  const int nv = (int)c->m->loc.n_vocab;
  if (c->tp_smp) tp_penalty_kernel<<<1, 256, 0, c->stream>>>(c->tp_smp, c->logits, nv, c->m->vocab0, c->tp_penalty);
  tp_argmax_kernel<<<1, 1024, 0, c->stream>>>(c->logits, nv, c->m->vocab0, best);
  if (c->tp_smp) tp_restore_kernel<<<1, 256, 0, c->stream>>>(c->tp_smp, c->logits, nv, c->m->vocab0);
  CK(cudaGetLastError(), "tp argmax");
  return FOXCUDA_OK;
}

// The next token from all shards' {value, index} pairs (on the device), the
// position advanced. The token stays in device memory for foxcuda_tp_embed
// (token -1) and is kept in the context's output ring.
extern "C" foxcuda_status foxcuda_tp_pick(foxcuda_context* c, const float* pairs) {
  foxcuda_status st = tp_check(c, 0, false);
  if (st) return st;
  if (!pairs) return fail(FOXCUDA_ERR_ARG, "tp_pick: null pairs");
  tp_pick_kernel<<<1, 32, 0, c->stream>>>(pairs, c->m->tp_size, c->token_dev, c->ring, (int)c->n_ctx,
                                          c->pos_dev);
  if (c->tp_smp) tp_accept_kernel<<<1, 32, 0, c->stream>>>(c->tp_smp, c->token_dev);
  advance_kernel<<<1, 32, 0, c->stream>>>(c->pos_dev, 1);
  CK(cudaGetLastError(), "tp pick");
  c->pos += 1;
  return FOXCUDA_OK;
}

// The next step's token from the host, for a captured step that embeds the
// token in device memory: one copy from pinned host memory on the context's
// stream (which is synchronised first, so the staging word is free).
extern "C" foxcuda_status foxcuda_tp_feed(foxcuda_context* c, uint32_t token) {
  if (!c) return fail(FOXCUDA_ERR_ARG, "tp_feed: null context");
  if (token >= c->m->info.n_vocab) return fail(FOXCUDA_ERR_ARG, "tp_feed: token outside the vocabulary");
  cudaSetDevice(c->m->device);
  CK(cudaStreamSynchronize(c->stream), "tp feed sync");
  c->h_pinned[0] = token;
  CK(cudaMemcpyAsync(c->token_dev, c->h_pinned, 4, cudaMemcpyHostToDevice, c->stream), "tp feed");
  return FOXCUDA_OK;
}

// Position advance without a pick (prompt tokens) and reading the picks back.
extern "C" foxcuda_status foxcuda_tp_advance(foxcuda_context* c) {
  foxcuda_status st = tp_check(c, 0, false);
  if (st) return st;
  // a prompt token's residual is not read again, but its completion is
  // what orders the next pushes (foxcuda_tp_embed)
  if ((st = flush_fold(c))) return st;
  advance_kernel<<<1, 32, 0, c->stream>>>(c->pos_dev, 1);
  CK(cudaGetLastError(), "tp advance");
  c->pos += 1;
  return FOXCUDA_OK;
}

// The host's position counter after graph replays advanced the device's.
extern "C" foxcuda_status foxcuda_context_sync_position(foxcuda_context* c) {
  if (!c) return fail(FOXCUDA_ERR_ARG, "sync_position: null context");
  cudaSetDevice(c->m->device);
  int p = 0;
  CK(cudaStreamSynchronize(c->stream), "sync");
  CK(cudaMemcpy(&p, c->pos_dev, 4, cudaMemcpyDeviceToHost), "position");
  c->pos = (uint32_t)p;
  return FOXCUDA_OK;
}

// This shard's logits of the last head evaluation (n floats to host).
extern "C" foxcuda_status foxcuda_context_logits(foxcuda_context* c, float* out, size_t n) {
  if (!c || !out) return fail(FOXCUDA_ERR_ARG, "logits: null argument");
  if (n > c->m->loc.n_vocab) return fail(FOXCUDA_ERR_ARG, "logits: %zu above %u", n, c->m->loc.n_vocab);
  cudaSetDevice(c->m->device);
  CK(cudaStreamSynchronize(c->stream), "logits sync");
  CK(cudaMemcpy(out, c->logits, n * 4, cudaMemcpyDeviceToHost), "logits copy");
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_tp_tokens(foxcuda_context* c, uint32_t first_pos, size_t n,
                                            uint32_t* out) {
  if (!c || !out) return fail(FOXCUDA_ERR_ARG, "tp_tokens: bad argument");
  cudaSetDevice(c->m->device);
  CK(cudaStreamSynchronize(c->stream), "tp sync");
  for (size_t i = 0; i < n; ++i)
    CK(cudaMemcpy(out + i, c->ring + (first_pos + i) % c->n_ctx, 4, cudaMemcpyDeviceToHost), "tp tokens");
  uint32_t code = 0;
  CK(cudaMemcpy(&code, c->err_dev, 4, cudaMemcpyDeviceToHost), "tp error word");
  if (code) {
    cudaMemset(c->err_dev, 0, 4);
    return fail(FOXCUDA_ERR_INTERNAL, "device: a bounded wait gave up (code %u: %s); the tokens are not valid",
                code, code == 2 ? "a peer's exchange did not arrive" : "weights did not reach shared memory");
  }
  return FOXCUDA_OK;
}

// Repeat penalty for the sharded greedy pick (upstream src/sample.c:95-107):
// each shard penalises the history tokens of its vocabulary rows before its
// argmax; the prompt tokens (foxcuda_tp_embed with a host token) and every
// pick enter the history. Set before the first step.
extern "C" foxcuda_status foxcuda_tp_set_penalty(foxcuda_context* c, float penalty, uint32_t last_n) {
  if (!c) return fail(FOXCUDA_ERR_ARG, "tp_set_penalty: null context");
  if (c->tp_smp) return fail(FOXCUDA_ERR_ARG, "tp_set_penalty: the penalty is already set");
  if (!(penalty >= 1.0f)) return fail(FOXCUDA_ERR_ARG, "tp_set_penalty: penalty %g is below 1", penalty);
  if (last_n > SAMPLER_MAX_HIST)
    return fail(FOXCUDA_ERR_UNSUPPORTED, "tp_set_penalty: repeat_last_n %u is above %d", last_n, SAMPLER_MAX_HIST);
  if (penalty == 1.0f) return FOXCUDA_OK;  // upstream skips the penalty at 1 (src/sample.c:98)
  cudaSetDevice(c->m->device);
  void* p = nullptr;
  CK(ctx_alloc(c, sizeof(SamplerDev), &p), "tp penalty state");
  CK(cudaMemset(p, 0, sizeof(SamplerDev)), "tp penalty state");
  const uint32_t cap = last_n ? last_n : 1;
  CK(cudaMemcpy(&reinterpret_cast<SamplerDev*>(p)->hist_cap, &cap, 4, cudaMemcpyHostToDevice), "tp penalty state");
  c->tp_smp = reinterpret_cast<SamplerDev*>(p);
  c->tp_penalty = penalty;
  return FOXCUDA_OK;
}

// ---- exchanges over peer memory (p2p.cuh) ------------------------------------

static uint32_t terms_per_block(int t) { return t == T_Q4_K ? 8u : t == T_Q6_K ? 4u : 1u; }

static XParams xparams(const foxcuda_context* c) {
  XParams x;
  memset(&x, 0, sizeof x);
  for (int k = 0; k < TPX_MAX; ++k) x.peers[k] = c->peer_arena[k];
  x.rank = c->m->tp_rank;
  x.world = c->m->tp_size;
  x.pos = c->pos_dev;
  x.err = c->err_dev;
  return x;
}

extern "C" foxcuda_status foxcuda_tp_p2p_export(foxcuda_context* c, void* handle) {
  if (!c || !handle) return fail(FOXCUDA_ERR_ARG, "tp_p2p_export: null argument");
  foxcuda_model* m = c->m;
  if (m->tp_size > TPX_MAX) return fail(FOXCUDA_ERR_UNSUPPORTED, "tp_p2p: at most %d shards", TPX_MAX);
  cudaSetDevice(m->device);
  if (!c->arena) {
    uint32_t to = 1, td = 1, fmax = 1;
    for (const LayerW& L : m->layers) {
      to = std::max(to, terms_per_block(L.o.type));
      td = std::max(td, terms_per_block(L.down.type));
    }
    for (int k = 0; k < m->tp_size; ++k) fmax = std::max(fmax, m->f_blocks_all[k]);
    c->stride_o = (int)(std::max(1u, m->o_blocks) * to);
    c->stride_d = (int)(fmax * td);
    const size_t E = m->info.n_embd;
    const size_t off_d = (AR_TERMS + E * (size_t)c->stride_o * 4 + 255) / 256 * 256;
    const size_t off_y = (off_d + E * (size_t)c->stride_d * 4 + 255) / 256 * 256;
    const size_t bytes = off_y + 2 * (size_t)m->tp_size * E * 8;
    c->y_off = off_y;
    void* p = nullptr;
    CK(ctx_alloc(c, bytes, &p), "exchange arena");
    CK(cudaMemset(p, 0, bytes), "exchange arena");
    c->arena = (uint8_t*)p;
    c->terms_d_off = off_d;
    CK(ctx_alloc(c, (4 + 2 * TPX_MAX) * 4, (void**)&c->x_small), "exchange scalars");
    CK(ctx_alloc(c, 2 * sizeof(unsigned), (void**)&c->x_count), "exchange counters");
  }
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, c->arena), "exchange handle");
  memcpy(handle, &h, sizeof h);
  return FOXCUDA_OK;
}

extern "C" foxcuda_status foxcuda_tp_p2p_open(foxcuda_context* c, const void* handles) {
  if (!c || !handles) return fail(FOXCUDA_ERR_ARG, "tp_p2p_open: null argument");
  if (!c->arena) return fail(FOXCUDA_ERR_ARG, "tp_p2p_open: export this context's arena first");
  if (c->p2p) return fail(FOXCUDA_ERR_ARG, "tp_p2p_open: the peers are already open");
  cudaSetDevice(c->m->device);
  for (int k = 0; k < c->m->tp_size; ++k) {
    if (k == c->m->tp_rank) {
      c->peer_arena[k] = c->arena;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, (const uint8_t*)handles + (size_t)k * sizeof h, sizeof h);
    void* p = nullptr;
    CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "open a peer's arena");
    c->peer_arena[k] = (uint8_t*)p;
    c->peer_ipc[k] = true;
  }
  c->p2p = true;
  return FOXCUDA_OK;
}

// The peers' arenas when every rank's context lives in this process (one
// process driving several GPUs, or several shards on one GPU): their device
// pointers, with peer access enabled between distinct devices.
extern "C" foxcuda_status foxcuda_tp_p2p_open_local(foxcuda_context* c, foxcuda_context* const* ranks) {
  if (!c || !ranks) return fail(FOXCUDA_ERR_ARG, "tp_p2p_open_local: null argument");
  if (!c->arena) return fail(FOXCUDA_ERR_ARG, "tp_p2p_open_local: export this context's arena first");
  if (c->p2p) return fail(FOXCUDA_ERR_ARG, "tp_p2p_open_local: the peers are already open");
  const foxcuda_model* m = c->m;
  for (int k = 0; k < m->tp_size; ++k) {
    const foxcuda_context* r = ranks[k];
    if (!r || !r->arena || r->m->tp_size != m->tp_size || r->m->tp_rank != k || r->n_ctx != c->n_ctx)
      return fail(FOXCUDA_ERR_ARG, "tp_p2p_open_local: entry %d is not an exported context of rank %d", k, k);
    if (k == m->tp_rank && r != c) return fail(FOXCUDA_ERR_ARG, "tp_p2p_open_local: entry %d is not this context", k);
  }
  cudaSetDevice(m->device);
  for (int k = 0; k < m->tp_size; ++k) {
    const int dev = ranks[k]->m->device;
    if (dev != m->device) {
      int can = 0;
      CK(cudaDeviceCanAccessPeer(&can, m->device, dev), "peer access query");
      if (!can) return fail(FOXCUDA_ERR_UNSUPPORTED, "tp_p2p_open_local: device %d cannot reach device %d", m->device, dev);
      const cudaError_t e = cudaDeviceEnablePeerAccess(dev, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
      else CK(e, "peer access");
    }
    c->peer_arena[k] = ranks[k]->arena;
  }
  c->p2p = true;
  return FOXCUDA_OK;
}

// Zero this rank's slots (after foxcuda_context_reset the epochs repeat).
// Every rank clears before any rank's next exchange.
extern "C" foxcuda_status foxcuda_tp_p2p_clear(foxcuda_context* c) {
  if (!c || !c->arena) return fail(FOXCUDA_ERR_ARG, "tp_p2p_clear: no arena");
  cudaSetDevice(c->m->device);
  CK(cudaStreamSynchronize(c->stream), "tp sync");
  CK(cudaMemset(c->arena, 0, AR_TERMS), "clear slots");
  CK(cudaMemset(c->x_count, 0, 2 * sizeof(unsigned)), "clear counters");
  return FOXCUDA_OK;
}

// The terms GEMV with both exchanges inside (gemv.cuh PRO_XAMAX, EPI_TERMS
// with the readiness count): ternary shards trade the absmax in the
// prologue; K-quant shards quantise with their own 256-block scales.
// With programmatic launch (FOXCUDA_TP_PDL=1) it takes the ring form, whose
// weight copies start before griddepcontrol.wait, so the shard's o or down
// weights stream while the attention or gate|up kernel still runs.
template <int T>
static cudaError_t launch_xterms_t(const GemvParams& p, cudaStream_t s) {
  constexpr int PRO = (T == T_TQ1_0 || T == T_TQ2_0) ? PRO_XAMAX : PRO_VEC;
  if (p.pdl) return launch_ring_t<T, PRO, EPI_TERMS>(p, s);
  return launch_gemv_t<T, PRO, EPI_TERMS>(p, s);
}

static cudaError_t launch_xterms(const foxcuda_context* c, const PackedMat& W, int which, int phase, float* amax,
                                 float* terms, int stride) {
  GemvParams p = gemv_base(W.type, W.dev, W.n_rows, W.K, W.nb, W.U);
  p.x = which == 0 ? c->att : c->h;
  p.out = terms;
  p.terms_stride = stride;
  p.pos = c->pos_dev;
  p.err = c->err_dev;
  for (int k = 0; k < TPX_MAX; ++k) p.x_peers[k] = c->peer_arena[k];
  p.x_rank = c->m->tp_rank;
  p.x_world = c->m->tp_size;
  p.x_which = which;
  p.x_phase = phase;
  p.x_count = c->x_count + which;
  p.x_amax = amax;
  p.pdl = ctx_pdl(c) ? 1 : 0;
  if (W.slice || W.stream) return launch_sliced(W, PRO_XAMAX, EPI_TERMS, p, c->stream);
  switch (W.type) {
    case T_TQ1_0: return launch_xterms_t<T_TQ1_0>(p, c->stream);
    case T_TQ2_0: return launch_xterms_t<T_TQ2_0>(p, c->stream);
    case T_Q4_K: return launch_xterms_t<T_Q4_K>(p, c->stream);
    case T_Q6_K: return launch_xterms_t<T_Q6_K>(p, c->stream);
    default: return cudaErrorInvalidValue;
  }
}

// The sums exchange's GEMV of one row-parallel projection: the absmax
// traded in the prologue (ternary; K-quant shards quantise with their own
// 256-block scales, which are the unsplit vector's), each row's value pushed
// to every rank as an {epoch, value} word (gemv.cuh EPI_XSUM).
static cudaError_t launch_xsum(const foxcuda_context* c, const PackedMat& W, int which, int phase) {
  const foxcuda_model* m = c->m;
  GemvParams p = gemv_base(W.type, W.dev, W.n_rows, W.K, W.nb, W.U);
  p.x = which == 0 ? c->att : c->h;
  p.pos = c->pos_dev;
  p.err = c->err_dev;
  for (int k = 0; k < TPX_MAX; ++k) p.x_peers[k] = c->peer_arena[k];
  p.x_rank = m->tp_rank;
  p.x_world = m->tp_size;
  p.x_which = which;
  p.x_phase = phase;
  p.x_y_off = c->y_off + (size_t)which * m->tp_size * m->info.n_embd * 8;
  p.x_res = c->x;
  p.pdl = ctx_pdl(c) ? 1 : 0;
  const bool tern = W.type == T_TQ1_0 || W.type == T_TQ2_0;
  const int pro = tern ? PRO_XAMAX : PRO_VEC;
  if (W.slice || W.stream) return launch_sliced(W, pro, EPI_XSUM, p, c->stream);
  return launch_ring(W.type, pro, EPI_XSUM, p, c->stream);
}

// A pending sums exchange completed into the residual by a GEMV's prologue
// (PRO_NFOLD): the exchange's area, readiness slot and phase.
static void set_nfold(const foxcuda_context* c, GemvParams& p) {
  const foxcuda_model* m = c->m;
  for (int k = 0; k < TPX_MAX; ++k) p.x_peers[k] = c->peer_arena[k];
  p.x_rank = m->tp_rank;
  p.x_world = m->tp_size;
  p.pos = c->pos_dev;
  p.f_y_off = c->y_off + (size_t)c->fold_which * m->tp_size * m->info.n_embd * 8;
  p.f_which = c->fold_which;
  p.f_phase = c->fold_phase;
  p.f_out = c->x;
}

// A pending sums exchange completed into the residual by a kernel of its own.
static cudaError_t enqueue_fold(foxcuda_context* c) {
  if (c->fold_which < 0) return cudaSuccess;
  const int E = (int)c->m->info.n_embd;
  const size_t y = c->y_off + (size_t)c->fold_which * c->m->tp_size * E * 8;
  fold_sum_x_kernel<<<(E + 255) / 256, 256, 0, c->stream>>>(xparams(c), y, c->fold_which, c->fold_phase, E, c->x);
  c->fold_which = -1;
  return cudaGetLastError();
}


// The row-parallel exchange of the steps that follow (every rank the same).
extern "C" foxcuda_status foxcuda_tp_p2p_mode(foxcuda_context* c, int mode) {
  if (!c) return fail(FOXCUDA_ERR_ARG, "tp_p2p_mode: null context");
  if (mode != FOXCUDA_TP_TERMS && mode != FOXCUDA_TP_SUMS)
    return fail(FOXCUDA_ERR_ARG, "tp_p2p_mode: mode %d is neither terms (0) nor sums (1)", mode);
  if (c->fold_which >= 0) return fail(FOXCUDA_ERR_ARG, "tp_p2p_mode: a step is half done");
  c->x_mode = mode;
  return FOXCUDA_OK;
}

// foxcuda_tp_amax + max-allreduce + foxcuda_tp_terms + all-gather +
// foxcuda_tp_fold, with the two exchanges over peer memory: the same values
// in the same order and no host collective. Two launches: the terms GEMV
// with both exchanges inside it, then the fold.
extern "C" foxcuda_status foxcuda_tp_p2p_row(foxcuda_context* c, uint32_t layer, int which) {
  foxcuda_status st = tp_check(c, layer, true);
  if (st) return st;
  if (!c->p2p) return fail(FOXCUDA_ERR_ARG, "tp_p2p_row: open the peers first");
  if (which != 0 && which != 1) return fail(FOXCUDA_ERR_ARG, "tp_p2p_row: which is 0 (o) or 1 (down)");
  const foxcuda_model* m = c->m;
  const PackedMat& W = which == 0 ? m->layers[layer].o : m->layers[layer].down;
  const bool tern = W.type == T_TQ1_0 || W.type == T_TQ2_0;
  const XParams x = xparams(c);
  const int phase = 2 * (int)layer + which + 1;
  if (c->x_mode == FOXCUDA_TP_SUMS) {
    if ((st = flush_fold(c))) return st;
    CK(launch_xsum(c, W, which, phase), "tp sums exchange");
    c->fold_which = which;
    c->fold_phase = phase;
    if (c->trace_on && which == 1) {  // the layer's output, as foxcuda_context_hidden reads it
      if ((st = flush_fold(c))) return st;
      CK(cudaMemcpyAsync(c->trace + (size_t)(layer + 1) * m->info.n_embd, c->x, m->info.n_embd * 4,
                         cudaMemcpyDeviceToDevice, c->stream), "trace");
    }
    return FOXCUDA_OK;
  }
  float* amax = c->x_small + which;
  const size_t off = which == 0 ? AR_TERMS : c->terms_d_off;
  const int stride = which == 0 ? c->stride_o : c->stride_d;
  CK(launch_xterms(c, W, which, phase, amax, (float*)(c->arena + off), stride), "tp terms exchange");
  FoldXParams f;
  memset(&f, 0, sizeof f);
  f.terms_off = off;
  f.rows = (int)m->info.n_embd;
  f.stride = stride;
  f.ternary = tern;
  f.which = which;
  f.phase = phase;
  const uint32_t nt = terms_per_block(W.type);
  for (int k = 0; k < m->tp_size; ++k) f.count[k] = (int)((which == 0 ? m->o_blocks : m->f_blocks_all[k]) * nt);
  f.amax = amax;
  f.x = c->x;
  fold_x_kernel<<<(f.rows + 255) / 256, 256, 0, c->stream>>>(x, f);
  CK(cudaGetLastError(), "tp fold exchange");
  if (c->trace_on && which == 1)
    CK(cudaMemcpyAsync(c->trace + (size_t)(layer + 1) * m->info.n_embd, c->x, m->info.n_embd * 4,
                       cudaMemcpyDeviceToDevice, c->stream), "trace");
  return FOXCUDA_OK;
}

// foxcuda_tp_head + all-gather of the pairs + foxcuda_tp_pick over peer memory.
extern "C" foxcuda_status foxcuda_tp_p2p_pick(foxcuda_context* c) {
  foxcuda_status st = tp_check(c, 0, false);
  if (st) return st;
  if (!c->p2p) return fail(FOXCUDA_ERR_ARG, "tp_p2p_pick: open the peers first");
  float* best = c->x_small + 2;
  float* pairs = c->x_small + 4;
  if ((st = foxcuda_tp_head(c, best))) return st;
  pick_x_kernel<<<1, 32, 0, c->stream>>>(xparams(c), best, pairs);
  CK(cudaGetLastError(), "tp pick exchange");
  return foxcuda_tp_pick(c, pairs);
}

// ---------------------------------------------------------------------------
// diagnostics

static void mark(foxcuda_context* c, int kind) {
  if (!c->prof) return;
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return;
  cudaEventRecord(e, c->stream);
  c->prof->push_back({e, kind});
}

extern "C" foxcuda_status foxcuda_context_profile(foxcuda_context* c, foxcuda_sampler* s,
                                                  uint32_t token, float* us, int* kinds, int cap,
                                                  int* n_out) {
  if (!c || !us || !kinds || !n_out || cap <= 0 || (s && s->c != c))
    return fail(FOXCUDA_ERR_ARG, "profile: bad argument");
  if (token >= c->m->info.n_vocab) return fail(FOXCUDA_ERR_ARG, "profile: token outside vocabulary");
  if (c->pos + 1 > c->n_ctx) return fail(FOXCUDA_ERR_ARG, "profile: context full");
  cudaSetDevice(c->m->device);
  std::vector<std::pair<cudaEvent_t, int>> marks;
  c->h_pinned[0] = token;
  CK(cudaMemcpyAsync(c->token_dev, c->h_pinned, 4, cudaMemcpyHostToDevice, c->stream), "token in");
  cudaEvent_t start;
  CK(cudaEventCreate(&start), "event");
  cudaEventRecord(start, c->stream);
  c->prof = &marks;
  cudaError_t e = enqueue_body(c, false);
  if (!e) e = enqueue_head(c);
  if (!e && s) e = enqueue_pick(s, true);
  c->prof = nullptr;
  enqueue_err_read(c);
  cudaError_t e2 = cudaStreamSynchronize(c->stream);
  int n = 0;
  cudaEvent_t prev = start;
  for (auto& mk : marks) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, prev, mk.first);
    if (n < cap) { us[n] = ms * 1e3f; kinds[n] = mk.second; ++n; }
    if (prev != start) cudaEventDestroy(prev);
    prev = mk.first;
  }
  if (prev != start) cudaEventDestroy(prev);
  cudaEventDestroy(start);
  *n_out = n;
  if (e) return cuda_fail(e, "profile");
  CK(e2, "profile");
  c->pos += 1;
  if (s) s->n_out += 1;
  return check_err(c);
}

extern "C" foxcuda_status foxcuda_context_bench_kernel(foxcuda_context* c, int kind, int reps,
                                                       double* us_per_launch,
                                                       uint64_t* weight_bytes_per_launch) {
  if (!c || !us_per_launch || !weight_bytes_per_launch || reps <= 0)
    return fail(FOXCUDA_ERR_ARG, "bench_kernel: bad argument");
  if (!(kind == PK_QKV || kind == PK_O || kind == PK_GATEUP || kind == PK_DOWN || kind == PK_HEAD))
    return fail(FOXCUDA_ERR_ARG, "bench_kernel: kind %d is not a weight GEMV", kind);
  cudaSetDevice(c->m->device);
  const uint32_t nl = c->m->info.n_layer;
  auto one = [&](int i) -> cudaError_t {
    const uint32_t l = (uint32_t)i % nl;  // successive layers: weights come from HBM
    switch (kind) {
      case PK_QKV: return launch_qkv(c, l);
      case PK_O: return launch_o(c, l);
      case PK_GATEUP: return launch_gateup(c, l);
      case PK_DOWN: return launch_down(c, l);
      default: return launch_head(c);
    }
  };
  for (int i = 0; i < 3; ++i) CK(one(i), "bench_kernel warm-up");
  CK(cudaEventRecord(c->ev0, c->stream), "event");
  for (int i = 0; i < reps; ++i) CK(one(i), "bench_kernel");
  CK(cudaEventRecord(c->ev1, c->stream), "event");
  enqueue_err_read(c);
  CK(cudaStreamSynchronize(c->stream), "bench_kernel");
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, c->ev0, c->ev1);
  uint64_t bytes = 0;
  for (int i = 0; i < reps; ++i) bytes += launch_weight_bytes(c->m, kind, (uint32_t)i % nl);
  *us_per_launch = ms * 1e3 / reps;
  *weight_bytes_per_launch = bytes / reps;
  return check_err(c);
}
