// Seeded synthetic weights generated on the device, for benchmark models too
// large to generate quickly on the host (the 27B shape: 9 GB per shard).
//
// Every byte is a pure function of (seed, block, field) through a splitmix64
// finalizer, so the result does not depend on the launch shape. The
// distributions are the synthetic configs': uniform ternary weights (TQ1_0,
// TQ2_0) and uniform K-quant bytes with fp16 block scales |N(0, sigma)|, and
// Q8_0 of N(0, sigma) values. Normals come from Box-Muller in double. The
// tests hold a numpy restatement of the same formulas.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace fox {

// counter stride per block (indices of one block never overlap the next)
constexpr uint64_t SG_TQ1 = 64, SG_TQ2 = 80, SG_Q8 = 48, SG_Q4K = 160, SG_Q6K = 224;

// a uniform integer in [0, n) from the high half of a hash
FOX_DEV uint32_t sg_below(uint64_t h, uint32_t n) { return (uint32_t)(((h >> 32) * n) >> 32); }

FOX_DEV uint64_t sg_mix(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// N(0, 1) pair from counters i and i + 1: sqrt(-2 ln u1) (cos, sin)(2 pi u2),
// u1 in (0, 1], u2 in [0, 1)
FOX_DEV void sg_normal2(uint64_t seed, uint64_t i, double& a, double& b) {
  const double u1 = ((double)(sg_mix(seed, i) >> 11) + 1.0) * 0x1.0p-53;
  const double u2 = (double)(sg_mix(seed, i + 1) >> 11) * 0x1.0p-53;
  const double r = sqrt(-2.0 * log(u1)), t = 6.283185307179586 * u2;
  a = r * cos(t);
  b = r * sin(t);
}

// fp16 bits of |z * sigma|, rounded to float, then to half
FOX_DEV uint16_t sg_half_abs(double z, double sigma) {
  return __half_as_ushort(__float2half_rn((float)fabs(z * sigma)));
}

FOX_DEV void sg_put16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)v;
  p[1] = (uint8_t)(v >> 8);
}

// one block of `type` (TQ1_0, TQ2_0, Q8_0, Q4_K, Q6_K) into o, block index b
FOX_DEV void sg_block_local(int type, uint8_t* o, uint64_t b, uint64_t seed, double sigma) {
  double z0, z1;
  if (type == T_TQ1_0) {
    // five uniform trits per qs byte (a uniform value in [0, 243)), four per
    // qh byte ([0, 81)), in the TQ1_0 byte encoding ceil(v * 256 / 3^k)
    const uint64_t base = b * SG_TQ1;
    for (int j = 0; j < 48; ++j) o[j] = (uint8_t)((sg_below(sg_mix(seed, base + j), 243) * 256u + 242u) / 243u);
    for (int j = 48; j < 52; ++j) o[j] = (uint8_t)((sg_below(sg_mix(seed, base + j), 81) * 256u + 80u) / 81u);
    sg_normal2(seed, base + 52, z0, z1);
    sg_put16(o + 52, sg_half_abs(z0, sigma));
  } else if (type == T_TQ2_0) {
    const uint64_t base = b * SG_TQ2;
    for (int j = 0; j < 64; ++j) {
      // a uniform choice among the 81 bytes of four codes in {0, 1, 2}
      const uint32_t c = sg_below(sg_mix(seed, base + j), 81);
      o[j] = (uint8_t)((c % 3) | ((c / 3 % 3) << 2) | ((c / 9 % 3) << 4) | ((c / 27) << 6));
    }
    sg_normal2(seed, base + 64, z0, z1);
    sg_put16(o + 64, sg_half_abs(z0, sigma));
  } else if (type == T_Q8_0) {
    const uint64_t base = b * SG_Q8;
    float x[32];
    for (int j = 0; j < 32; j += 2) {
      sg_normal2(seed, base + j, z0, z1);
      x[j] = (float)(z0 * sigma);
      x[j + 1] = (float)(z1 * sigma);
    }
    // round-to-nearest Q8_0: d = amax / 127 as fp16, q = rint(x / d)
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
    const __half d = __float2half_rn(__fdiv_rn(amax, 127.0f));
    const float df = __half2float(d);
    const float inv = df > 0.0f ? __fdiv_rn(1.0f, df) : 0.0f;
    sg_put16(o, __half_as_ushort(d));
    for (int j = 0; j < 32; ++j) {
      const float q = fminf(fmaxf(rintf(__fmul_rn(x[j], inv)), -127.0f), 127.0f);
      o[2 + j] = (uint8_t)(int8_t)q;
    }
  } else if (type == T_Q4_K) {
    const uint64_t base = b * SG_Q4K;
    for (int j = 4; j < 144; ++j) o[j] = (uint8_t)(sg_mix(seed, base + j) >> 56);
    sg_normal2(seed, base + 144, z0, z1);
    sg_put16(o, sg_half_abs(z0, sigma));      // d
    sg_put16(o + 2, sg_half_abs(z1, sigma));  // dmin
  } else if (type == T_Q6_K) {
    const uint64_t base = b * SG_Q6K;
    for (int j = 0; j < 208; ++j) o[j] = (uint8_t)(sg_mix(seed, base + j) >> 56);
    sg_normal2(seed, base + 208, z0, z1);
    sg_put16(o + 208, sg_half_abs(z0, sigma));
  }
}

// The block is formed in a local array and then stored byte by byte: storing
// the fp16 scale straight into the block's global bytes lost its low byte on
// the device (measured: the high byte right, the low byte zero), while the
// same value formed locally is right.
__global__ void synth_fill_kernel(int type, uint8_t* out, long n_blocks, int block_bytes, uint64_t seed,
                                  double sigma) {
  for (long b = blockIdx.x * (long)blockDim.x + threadIdx.x; b < n_blocks; b += (long)gridDim.x * blockDim.x) {
    uint8_t blk[224];
    sg_block_local(type, blk, (uint64_t)b, seed, sigma);
    uint8_t* o = out + b * block_bytes;
    for (int i = 0; i < block_bytes; ++i) o[i] = blk[i];
  }
}

}  // namespace fox
