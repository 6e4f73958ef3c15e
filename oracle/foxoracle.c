/*
 * foxoracle.c -- CPU restatement of RustFox's token loop. TEST INFRASTRUCTURE
 * ONLY (see foxoracle.h): the parity checker, never the thing measured or
 * shipped. Built with -ffp-contract=off so each float operation rounds once,
 * in the order the upstream C source writes it.
 */
#include "foxoracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static __thread char g_err[256];

static int fail(int st, const char *msg)
{
    snprintf(g_err, sizeof(g_err), "%s", msg);
    return st;
}

const char *or_last_error(void) { return g_err[0] ? g_err : "no error recorded"; }

/* Upstream calls libm's expf (src/ops.c:32,46, src/sample.c:165), and so
 * does the oracle by default; the device computes the same function (glibc's
 * algorithm, restated in CUDA). glibc's expf is not correctly rounded: it
 * differs from the correctly rounded e^x on about 7.6e-5 of the inputs in
 * [-104, 89]. Mode 1 swaps in the correctly rounded value,
 * (float)exp((double)x), to show what that difference alone changes. */
static int g_exp_cr = 0;

void or_set_exp_mode(int correctly_rounded) { g_exp_cr = correctly_rounded != 0; }

static float or_expf(float x) { return g_exp_cr ? (float)exp((double)x) : expf(x); }

/* Test support: how many of got[i] differ (bit for bit) from libm's expf of
 * the float whose bit pattern is first_bits + i; the first such i in
 * *first_bad (n when none). */
size_t or_expf_mismatches(uint32_t first_bits, size_t n, const float *got, size_t *first_bad)
{
    size_t bad = 0, first = n;
    for (size_t i = 0; i < n; ++i) {
        const uint32_t b = first_bits + (uint32_t)i;
        float x, want;
        memcpy(&x, &b, 4);
        want = expf(x);
        if (memcmp(&want, &got[i], 4) != 0) {
            if (first == n) first = i;
            ++bad;
        }
    }
    if (first_bad) *first_bad = first;
    return bad;
}

/* ---- element conversion ------------------------------------------------ */

/* upstream src/kernels.c:14-39 (also src/ternary.c:26-51): exact binary16 ->
 * binary32, subnormals included. Restated with the subnormal computed as an
 * exact power-of-two product instead of a normalisation loop. */
float or_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1Fu, f = h & 0x3FFu;
    union { uint32_t u; float f; } v;
    if (e == 0) {
        float mag = (float)f * 5.9604644775390625e-8f; /* f * 2^-24, exact */
        v.f = mag;
        v.u |= sign;
        return v.f;
    }
    if (e == 31) { v.u = sign | 0x7F800000u | (f << 13); return v.f; }
    v.u = sign | ((e + 112u) << 23) | (f << 13);
    return v.f;
}

/* binary32 -> binary16, IEEE round-to-nearest-even (the rounding CUDA's
 * __float2half_rn applies). Used only for the fp16 KV-cache mode. */
uint16_t or_f32_to_f16_rne(float x)
{
    union { float f; uint32_t u; } v;
    uint32_t sign, absu, mant;
    int e;
    v.f = x;
    sign = (v.u >> 16) & 0x8000u;
    absu = v.u & 0x7FFFFFFFu;
    if (absu >= 0x7F800000u)
        return (uint16_t)(sign | 0x7C00u | (absu > 0x7F800000u ? 0x200u : 0u));
    if (absu >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to inf */
    e = (int)(absu >> 23) - 127;
    if (e >= -14) {                                  /* normal half */
        uint32_t m = absu & 0x7FFFFFu;
        uint32_t out = ((uint32_t)(e + 15) << 10) | (m >> 13);
        uint32_t rem = m & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (out & 1u))) out++;
        return (uint16_t)(sign | out);
    }
    if (e < -25) return (uint16_t)sign;              /* below half of min subnormal */
    mant = (absu & 0x7FFFFFu) | 0x800000u;           /* subnormal half */
    {
        int shift = -e - 14 + 13;                    /* 14..24 */
        uint32_t out = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (out & 1u))) out++;
        return (uint16_t)(sign | out);
    }
}

static uint16_t le16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static float half_at(const uint8_t *p) { return or_f16_to_f32(le16(p)); }

/* block geometry, upstream src/gguf.c:160-195 */
static int layout(int type, size_t *blk, size_t *bytes)
{
    switch (type) {
    case OR_F32:  *blk = 1;   *bytes = 4;   return 1;
    case OR_F16:  *blk = 1;   *bytes = 2;   return 1;
    case OR_Q8_0: *blk = 32;  *bytes = 34;  return 1;
    case OR_Q4_K: *blk = 256; *bytes = 144; return 1;
    case OR_Q6_K: *blk = 256; *bytes = 210; return 1;
    case OR_TQ1_0:*blk = 256; *bytes = 54;  return 1;
    case OR_TQ2_0:*blk = 256; *bytes = 66;  return 1;
    default: return 0;
    }
}

/* upstream src/kernels.c:690-698 */
size_t or_row_bytes(int type, size_t n_cols)
{
    size_t blk, bytes;
    if (!layout(type, &blk, &bytes) || n_cols % blk) return 0;
    return n_cols / blk * bytes;
}

/* ---- activation quantisers --------------------------------------------- */

/* one int8 value with upstream's rounding: half away from zero, then clamp
 * (src/gemv.c:113-119, src/kernels.c:745-751) */
static int8_t q_round(float x, float inv)
{
    float v = x * inv;
    int r = (int)(v < 0.0f ? v - 0.5f : v + 0.5f);
    if (r > 127) r = 127;
    if (r < -127) r = -127;
    return (int8_t)r;
}

static float abs_max(const float *x, size_t n)
{
    float amax = 0.0f;
    size_t i;
    for (i = 0; i < n; i++) {
        float a = x[i] < 0.0f ? -x[i] : x[i];
        if (a > amax) amax = a;
    }
    return amax;
}

/* upstream src/gemv.c:11-42: one absmax scale for the whole vector */
int or_quantize_i8(const float *x, size_t n, int8_t *q, float *scale)
{
    float amax, inv;
    size_t i;
    if (!x || !q || !scale || n == 0) return OR_ERR_ARG;
    amax = abs_max(x, n);
    if (!(amax > 0.0f)) { memset(q, 0, n); *scale = 0.0f; return OR_OK; }
    inv = 127.0f / amax;
    for (i = 0; i < n; i++) q[i] = q_round(x[i], inv);
    *scale = amax / 127.0f;
    return OR_OK;
}

/* upstream src/kernels.c:722-754: one absmax scale per 256-element block */
int or_quantize_k(const float *x, size_t n, int8_t *q, float *scales)
{
    size_t b, i;
    if (!x || !q || !scales || n == 0 || n % 256) return OR_ERR_ARG;
    for (b = 0; b < n / 256; b++) {
        float amax = abs_max(x + b * 256, 256), inv;
        if (!(amax > 0.0f)) { memset(q + b * 256, 0, 256); scales[b] = 0.0f; continue; }
        inv = 127.0f / amax;
        for (i = 0; i < 256; i++) q[b * 256 + i] = q_round(x[b * 256 + i], inv);
        scales[b] = amax / 127.0f;
    }
    return OR_OK;
}

/* ---- ternary blocks ---------------------------------------------------- */

/* upstream src/ternary.c:59-63: level l of a base-3 byte is
 * ((code * 3^l mod 256) * 3) >> 8, shifted to {-1, 0, +1} */
static int trit(uint8_t code, int level)
{
    static const uint8_t p3[5] = { 1, 3, 9, 27, 81 };
    uint32_t q = (uint8_t)(code * p3[level]);
    return (int)((q * 3u) >> 8) - 1;
}

/* upstream src/ternary.c:73-93 (TQ1_0, 54 B: qs[48], qh[4], fp16 d).
 * Element l*32+m is qs[m] level l; 160 + l*16 + m is qs[32+m] level l;
 * 240 + l*4 + m is qh[m] level l. */
int32_t or_tq1_block_sum(const int8_t *x, const uint8_t *b)
{
    int32_t s = 0;
    int l, m;
    for (l = 0; l < 5; l++)
        for (m = 0; m < 32; m++) s += trit(b[m], l) * x[l * 32 + m];
    for (l = 0; l < 5; l++)
        for (m = 0; m < 16; m++) s += trit(b[32 + m], l) * x[160 + l * 16 + m];
    for (l = 0; l < 4; l++)
        for (m = 0; m < 4; m++) s += trit(b[48 + m], l) * x[240 + l * 4 + m];
    return s;
}

/* upstream src/ternary.c:177-188 (TQ2_0, 66 B: qs[64], fp16 d). Element
 * j*128 + l*32 + m is ((qs[j*32+m] >> 2l) & 3) - 1. */
int32_t or_tq2_block_sum(const int8_t *x, const uint8_t *qs)
{
    int32_t s = 0;
    int j, l, m;
    for (j = 0; j < 2; j++)
        for (l = 0; l < 4; l++)
            for (m = 0; m < 32; m++)
                s += (((qs[j * 32 + m] >> (2 * l)) & 3) - 1) * x[j * 128 + l * 32 + m];
    return s;
}

/* upstream src/ternary.c:226-246 + src/gemv.c:54-72: per row, the fp16 block
 * scale times the int32 block sum accumulates in block order from 0.0f, then
 * the row total is multiplied by the vector's activation scale. */
int or_gemv_tq_i8(int type, const int8_t *q, float act_scale, const void *w,
                  size_t n_rows, size_t n_cols, float *out)
{
    size_t bb = type == OR_TQ1_0 ? 54 : 66, nb;
    long r;
    if (type != OR_TQ1_0 && type != OR_TQ2_0) return fail(OR_ERR_UNSUPPORTED, "not ternary");
    if (!q || !w || !out || n_rows == 0 || n_cols == 0) return OR_ERR_ARG;
    if (n_cols % 256) return fail(OR_ERR_ARG, "gemv: columns not a multiple of 256");
    nb = n_cols / 256;
#pragma omp parallel for schedule(static)
    for (r = 0; r < (long)n_rows; r++) {
        const uint8_t *row = (const uint8_t *)w + (size_t)r * nb * bb;
        float acc = 0.0f;
        size_t b;
        for (b = 0; b < nb; b++) {
            const uint8_t *blk = row + b * bb;
            int32_t s = type == OR_TQ1_0 ? or_tq1_block_sum(q + b * 256, blk)
                                         : or_tq2_block_sum(q + b * 256, blk);
            acc += half_at(blk + bb - 2) * (float)s;
        }
        out[r] = acc * act_scale;
    }
    return OR_OK;
}

/* ---- K-quant blocks ---------------------------------------------------- */

/* upstream src/kernels.c:246-255: 6-bit scale and min of sub-block j */
static void scale_min(int j, const uint8_t *s, int *d, int *m)
{
    if (j < 4) { *d = s[j] & 63; *m = s[j + 4] & 63; }
    else {
        *d = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Q4_K sub-block j (32 elements) of a 144-byte block: integer dot of the
 * nibbles with q and the plain sum of q (upstream src/kernels.c:465-500) */
static void q4k_sub(const uint8_t *blk, const int8_t *xb, int j, int32_t *dot, int32_t *sum)
{
    const uint8_t *qs = blk + 16 + (j / 2) * 32;
    const int8_t *x = xb + j * 32;
    int l, hi = j & 1;
    *dot = 0; *sum = 0;
    for (l = 0; l < 32; l++) {
        int nib = hi ? (qs[l] >> 4) : (qs[l] & 0x0F);
        *dot += nib * x[l];
        *sum += x[l];
    }
}

/* Q6_K (half, sub) group of a 210-byte block: sum over the four 16-element
 * runs of the int8 scale times the signed 6-bit dot (upstream
 * src/kernels.c:531-569) */
static int32_t q6k_group(const uint8_t *blk, const int8_t *xb, int half, int sub)
{
    const uint8_t *ql = blk + half * 64, *qh = blk + 128 + half * 32;
    const int8_t *sc = (const int8_t *)(blk + 192) + half * 8;
    const int8_t *x = xb + half * 128;
    int32_t d0 = 0, d1 = 0, d2 = 0, d3 = 0;
    int l;
    for (l = sub * 16; l < sub * 16 + 16; l++) {
        int q0 = ((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
        int q1 = ((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
        int q2 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
        int q3 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
        d0 += q0 * x[l]; d1 += q1 * x[l + 32]; d2 += q2 * x[l + 64]; d3 += q3 * x[l + 96];
    }
    return sc[sub] * d0 + sc[sub + 2] * d1 + sc[sub + 4] * d2 + sc[sub + 6] * d3;
}

/* upstream src/kernels.c:571-602: row dot of a Q4_K row with per-256 int8
 * activations, float terms accumulated in sub-block order */
static float q4k_row(const uint8_t *w, const int8_t *x, size_t n, const float *as)
{
    float sum = 0.0f;
    size_t b;
    for (b = 0; b < n / 256; b++) {
        const uint8_t *blk = w + b * 144;
        float d = half_at(blk), dmin = half_at(blk + 2);
        int j;
        for (j = 0; j < 8; j++) {
            int sc, m;
            int32_t dot, s;
            scale_min(j, blk + 4, &sc, &m);
            q4k_sub(blk, x + b * 256, j, &dot, &s);
            sum += as[b] * (d * (float)sc * (float)dot - dmin * (float)m * (float)s);
        }
    }
    return sum;
}

/* upstream src/kernels.c:636-661 */
static float q6k_row(const uint8_t *w, const int8_t *x, size_t n, const float *as)
{
    float sum = 0.0f;
    size_t b;
    for (b = 0; b < n / 256; b++) {
        const uint8_t *blk = w + b * 210;
        float d = half_at(blk + 208);
        int half, sub;
        for (half = 0; half < 2; half++)
            for (sub = 0; sub < 2; sub++)
                sum += as[b] * d * (float)q6k_group(blk, x + b * 256, half, sub);
    }
    return sum;
}

/* upstream src/kernels.c:98-113: Q8_0 row against FLOAT activations */
static float q8_0_row(const uint8_t *w, const float *x, size_t n)
{
    float sum = 0.0f;
    size_t b, j;
    for (b = 0; b < n / 32; b++) {
        const uint8_t *blk = w + b * 34;
        const int8_t *qs = (const int8_t *)(blk + 2);
        float d = half_at(blk), acc = 0.0f;
        for (j = 0; j < 32; j++) acc += (float)qs[j] * x[b * 32 + j];
        sum += d * acc;
    }
    return sum;
}

/* upstream src/kernels.c:81-96 */
static float f32_row(const uint8_t *w, const float *x, size_t n)
{
    const float *fw = (const float *)(const void *)w;
    float sum = 0.0f;
    size_t i;
    for (i = 0; i < n; i++) sum += fw[i] * x[i];
    return sum;
}

static float f16_row(const uint8_t *w, const float *x, size_t n)
{
    float sum = 0.0f;
    size_t i;
    for (i = 0; i < n; i++) sum += half_at(w + 2 * i) * x[i];
    return sum;
}

int or_block_partials(int type, const int8_t *q, const void *w,
                      size_t n_rows, size_t n_cols, int32_t *out)
{
    size_t rb = or_row_bytes(type, n_cols), nb = n_cols / 256, r, b;
    if (!q || !w || !out || rb == 0 || n_cols % 256) return OR_ERR_ARG;
    for (r = 0; r < n_rows; r++) {
        const uint8_t *row = (const uint8_t *)w + r * rb;
        for (b = 0; b < nb; b++) {
            const int8_t *xb = q + b * 256;
            if (type == OR_TQ1_0) {
                out[r * nb + b] = or_tq1_block_sum(xb, row + b * 54);
            } else if (type == OR_TQ2_0) {
                out[r * nb + b] = or_tq2_block_sum(xb, row + b * 66);
            } else if (type == OR_Q4_K) {
                int j;
                for (j = 0; j < 8; j++)
                    q4k_sub(row + b * 144, xb, j, &out[(r * nb + b) * 16 + 2 * j],
                            &out[(r * nb + b) * 16 + 2 * j + 1]);
            } else if (type == OR_Q6_K) {
                int g;
                for (g = 0; g < 4; g++)
                    out[(r * nb + b) * 4 + g] = q6k_group(row + b * 210, xb, g / 2, g % 2);
            } else {
                return fail(OR_ERR_UNSUPPORTED, "no integer partials for this type");
            }
        }
    }
    return OR_OK;
}

/* upstream src/kernels.c:809-872 with its x86 dispatch: ternary types go
 * through the per-vector int8 quantiser, Q4_K/Q6_K through the per-256 int8
 * quantiser, Q8_0/F32/F16 take float activations. */
int or_gemv(int type, const float *x, const void *w, size_t n_rows,
            size_t n_cols, float *out)
{
    size_t rb;
    long r;
    if (!x || !w || !out || n_rows == 0 || n_cols == 0) return OR_ERR_ARG;
    if (type == OR_TQ1_0 || type == OR_TQ2_0) {
        int8_t *q = (int8_t *)malloc(n_cols);
        float scale = 0.0f;
        int st;
        if (!q) return OR_ERR_ARG;
        st = or_quantize_i8(x, n_cols, q, &scale);
        if (st == OR_OK) st = or_gemv_tq_i8(type, q, scale, w, n_rows, n_cols, out);
        free(q);
        return st;
    }
    rb = or_row_bytes(type, n_cols);
    if (type != OR_Q4_K && type != OR_Q6_K && type != OR_Q8_0 &&
        type != OR_F32 && type != OR_F16)
        return fail(OR_ERR_UNSUPPORTED, "gemv: type not covered");
    if (rb == 0) return fail(OR_ERR_ARG, "gemv: ragged column count");
    if (type == OR_Q4_K || type == OR_Q6_K) {
        int8_t *q = (int8_t *)malloc(n_cols);
        float *as = (float *)malloc(n_cols / 256 * sizeof(float));
        if (!q || !as) { free(q); free(as); return OR_ERR_ARG; }
        or_quantize_k(x, n_cols, q, as);
#pragma omp parallel for schedule(static)
        for (r = 0; r < (long)n_rows; r++) {
            const uint8_t *row = (const uint8_t *)w + (size_t)r * rb;
            out[r] = type == OR_Q4_K ? q4k_row(row, q, n_cols, as)
                                     : q6k_row(row, q, n_cols, as);
        }
        free(q); free(as);
        return OR_OK;
    }
#pragma omp parallel for schedule(static)
    for (r = 0; r < (long)n_rows; r++) {
        const uint8_t *row = (const uint8_t *)w + (size_t)r * rb;
        out[r] = type == OR_Q8_0 ? q8_0_row(row, x, n_cols)
               : type == OR_F32  ? f32_row(row, x, n_cols)
                                 : f16_row(row, x, n_cols);
    }
    return OR_OK;
}

/* upstream src/kernels.c:874-941 (the types this build covers) */
int or_dequant_row(int type, const void *row, size_t n, float *out)
{
    const uint8_t *w = (const uint8_t *)row;
    size_t i, b;
    if (!row || !out || n == 0) return OR_ERR_ARG;
    if (or_row_bytes(type, n) == 0) return fail(OR_ERR_ARG, "dequant: ragged");
    switch (type) {
    case OR_F32: memcpy(out, w, n * 4); return OR_OK;
    case OR_F16: for (i = 0; i < n; i++) out[i] = half_at(w + 2 * i); return OR_OK;
    case OR_Q8_0:
        for (b = 0; b < n / 32; b++) {
            float d = half_at(w + b * 34);
            for (i = 0; i < 32; i++) out[b * 32 + i] = (float)(int8_t)w[b * 34 + 2 + i] * d;
        }
        return OR_OK;
    case OR_Q4_K:   /* upstream src/kernels.c:257-283 */
        for (b = 0; b < n / 256; b++) {
            const uint8_t *blk = w + b * 144;
            float d = half_at(blk), dmin = half_at(blk + 2);
            int j, l;
            for (j = 0; j < 8; j++) {
                int sc, m;
                float d1, m1;
                const uint8_t *qs = blk + 16 + (j / 2) * 32;
                scale_min(j, blk + 4, &sc, &m);
                d1 = d * (float)sc;
                m1 = dmin * (float)m;
                for (l = 0; l < 32; l++) {
                    int nib = (j & 1) ? (qs[l] >> 4) : (qs[l] & 0x0F);
                    out[b * 256 + j * 32 + l] = d1 * (float)nib - m1;
                }
            }
        }
        return OR_OK;
    case OR_Q6_K:   /* upstream src/kernels.c:217-244 */
        for (b = 0; b < n / 256; b++) {
            const uint8_t *blk = w + b * 210;
            float d = half_at(blk + 208);
            int e;
            for (e = 0; e < 256; e++) {
                int half = e / 128, grp = (e % 128) / 32, l = e % 32;
                const uint8_t *ql = blk + half * 64, *qh = blk + 128 + half * 32;
                const int8_t *sc = (const int8_t *)(blk + 192) + half * 8;
                int lo = (grp & 1) ? ql[l + 32] : ql[l];
                int q;
                lo = (grp & 2) ? (lo >> 4) : (lo & 0x0F);
                q = (lo | (((qh[l] >> (2 * grp)) & 3) << 4)) - 32;
                out[b * 256 + e] = d * (float)sc[l / 16 + 2 * grp] * (float)q;
            }
        }
        return OR_OK;
    default:
        return fail(OR_ERR_UNSUPPORTED, "dequant: type not covered");
    }
}

/* ---- element-wise ops, upstream src/ops.c ------------------------------- */

/* src/ops.c:7-22: sum of squares in double */
void or_rmsnorm(float *out, const float *x, const float *w, size_t n, float eps)
{
    double sum = 0.0;
    float scale;
    size_t i;
    for (i = 0; i < n; i++) sum += (double)x[i] * (double)x[i];
    scale = (float)(1.0 / sqrt(sum / (double)n + (double)eps));
    for (i = 0; i < n; i++) out[i] = w ? x[i] * scale * w[i] : x[i] * scale;
}

/* src/ops.c:24-39 */
void or_softmax(float *x, size_t n)
{
    float mx = x[0], sum = 0.0f;
    size_t i;
    for (i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    for (i = 0; i < n; i++) { x[i] = or_expf(x[i] - mx); sum += x[i]; }
    if (sum > 0.0f) {
        float inv = 1.0f / sum;
        for (i = 0; i < n; i++) x[i] *= inv;
    }
}

/* src/ops.c:41-48 */
void or_silu_mul(float *gate, const float *up, size_t n)
{
    size_t i;
    for (i = 0; i < n; i++) {
        float g = gate[i];
        gate[i] = (g / (1.0f + or_expf(-g))) * up[i];
    }
}

/* src/ops.c:50-54 */
void or_add(float *dst, const float *src, size_t n)
{
    size_t i;
    for (i = 0; i < n; i++) dst[i] += src[i];
}

/* src/ops.c:56-73: rotation of adjacent pairs (2i, 2i+1) */
void or_rope(float *v, size_t n_heads, size_t hd, const float *c, const float *s)
{
    size_t h, i;
    for (h = 0; h < n_heads; h++)
        for (i = 0; i < hd / 2; i++) {
            float *p = v + h * hd + 2 * i, x0 = p[0], x1 = p[1];
            p[0] = x0 * c[i] - x1 * s[i];
            p[1] = x0 * s[i] + x1 * c[i];
        }
}

/* src/ops.c:75-81 */
float or_dot_f32(const float *a, const float *b, size_t n)
{
    float s = 0.0f;
    size_t i;
    for (i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

/* ---- the forward pass, upstream src/forward.c ------------------------- */

struct or_ctx {
    const or_model *m;
    uint32_t n_ctx, pos;
    int kv_mode;
    int attn_nt;        /* 0: upstream's serial attention; > 0: the tile attention */
    float *tile_o;      /* the tile attention's per-tile sums [nt][head_dim] */
    size_t nq, nkv, wide;
    float *kc, *vc, *x, *xb, *xb2, *q, *k, *v, *hb, *hb2, *att, *norm, *rc, *rs;
};

or_ctx *or_ctx_create(const or_model *m, uint32_t n_ctx, int kv_mode)
{
    const or_model_info *mi = &m->info;
    or_ctx *c = (or_ctx *)calloc(1, sizeof(*c));
    size_t half = mi->head_dim / 2, p, i;
    if (!c) return NULL;
    c->m = m; c->n_ctx = n_ctx; c->kv_mode = kv_mode;
    c->nq = (size_t)mi->n_head * mi->head_dim;              /* forward.c:81-84 */
    c->nkv = (size_t)mi->n_head_kv * mi->head_dim;
    c->wide = c->nq > mi->n_embd ? c->nq : mi->n_embd;
    c->kc = (float *)calloc((size_t)mi->n_layer * n_ctx * c->nkv, 4);
    c->vc = (float *)calloc((size_t)mi->n_layer * n_ctx * c->nkv, 4);
    c->x = (float *)calloc(mi->n_embd, 4);
    c->xb = (float *)calloc(c->wide, 4);
    c->xb2 = (float *)calloc(c->wide, 4);
    c->q = (float *)calloc(c->nq, 4);
    c->k = (float *)calloc(c->nkv, 4);
    c->v = (float *)calloc(c->nkv, 4);
    c->hb = (float *)calloc(mi->n_ff, 4);
    c->hb2 = (float *)calloc(mi->n_ff, 4);
    c->att = (float *)calloc(n_ctx, 4);
    c->norm = (float *)calloc(c->wide, 4);
    c->rc = (float *)calloc((size_t)n_ctx * half, 4);
    c->rs = (float *)calloc((size_t)n_ctx * half, 4);
    if (!c->kc || !c->vc || !c->x || !c->xb || !c->xb2 || !c->q || !c->k ||
        !c->v || !c->hb || !c->hb2 || !c->att || !c->norm || !c->rc || !c->rs) {
        or_ctx_destroy(c);
        return NULL;
    }
    for (p = 0; p < n_ctx; p++)                             /* forward.c:107-118 */
        for (i = 0; i < half; i++) {
            double th = (double)p * pow((double)mi->rope_freq_base,
                                        -2.0 * (double)i / (double)mi->head_dim);
            c->rc[p * half + i] = (float)cos(th);
            c->rs[p * half + i] = (float)sin(th);
        }
    return c;
}

int or_ctx_set_attn_tiles(or_ctx *c, int nt)
{
    if (!c || nt < 0 || nt > 64) return fail(OR_ERR_ARG, "attention tiles: 0..64");
    free(c->tile_o);
    c->tile_o = NULL;
    c->attn_nt = nt;
    if (nt > 0) {
        c->tile_o = (float *)calloc((size_t)nt * c->m->info.head_dim, 4);
        if (!c->tile_o) return fail(OR_ERR_ARG, "attention tiles: out of memory");
    }
    return OR_OK;
}

void or_ctx_destroy(or_ctx *c)
{
    if (!c) return;
    free(c->tile_o);
    free(c->kc); free(c->vc); free(c->x); free(c->xb); free(c->xb2); free(c->q);
    free(c->k); free(c->v); free(c->hb); free(c->hb2); free(c->att); free(c->norm);
    free(c->rc); free(c->rs); free(c);
}

void or_ctx_reset(or_ctx *c) { if (c) c->pos = 0; }
uint32_t or_ctx_pos(const or_ctx *c) { return c ? c->pos : 0; }

static int project(const or_tensor *t, const float *in, float *out)
{
    return or_gemv(t->type, in, t->data, (size_t)t->ne1, (size_t)t->ne0, out);
}

static int norm_w(or_ctx *c, const or_tensor *t, const float **w)
{
    int st = or_dequant_row(t->type, t->data, c->m->info.n_embd, c->norm);
    *w = c->norm;
    return st;
}

static float kv_round(const or_ctx *c, float v)
{
    return c->kv_mode ? or_f16_to_f32(or_f32_to_f16_rne(v)) : v;
}

/* libfoxcuda's tile attention (rustfox_b200/csrc/attn.cuh) for one query head
 * over positions 0..P-1 of one KV head (rows `stride` floats apart). This is
 * not upstream's order; it is the production mode of the device, restated so
 * that mode is checked bit for bit. Positions are cut into tiles of
 * T = ceil(P / nt). Per tile: every score is the sum of 32
 * lane partials (hd/32 dimensions each: q0*k0, then fmaf in dimension order)
 * by an xor butterfly, times scale; the tile's max; e = exp(s - max); the sum
 * of e in ascending order; and per dimension fmaf(e, v, .) in ascending
 * order. The tiles are merged in order with weights exp(m_t - M): fmaf of
 * the sums, fmaf of the outputs, one division. */
static void tile_attention_into(const float *qh, const float *K, const float *V, size_t stride,
                                size_t hd, size_t P, int nt_target, float scale, float *out,
                                float *sc, float *tile_o)
{
    const size_t nt = (size_t)nt_target, T = (P + nt - 1) / nt;
    const size_t ntl = (P + T - 1) / T, dpl = hd / 32;
    float m[64], l[64], w[64], M = -INFINITY, L = 0.0f;
    size_t t, j, d, i, lane, off;
    for (t = 0; t < ntl; t++) {
        const size_t j0 = t * T, n = (P - j0 < T) ? P - j0 : T;
        float mx = -INFINITY, lt = 0.0f;
        for (j = 0; j < n; j++) {
            const float *k = K + (j0 + j) * stride;
            float p[32], np[32];
            for (lane = 0; lane < 32; lane++) {
                const float *qa = qh + lane * dpl, *ka = k + lane * dpl;
                float a = qa[0] * ka[0];
                for (i = 1; i < dpl; i++) a = fmaf(qa[i], ka[i], a);
                p[lane] = a;
            }
            for (off = 16; off > 0; off >>= 1) {
                for (lane = 0; lane < 32; lane++) np[lane] = p[lane] + p[lane ^ off];
                memcpy(p, np, sizeof(p));
            }
            sc[j] = p[0] * scale;
        }
        for (j = 0; j < n; j++) mx = fmaxf(mx, sc[j]);
        for (j = 0; j < n; j++) sc[j] = or_expf(sc[j] - mx);
        for (j = 0; j < n; j++) lt = lt + sc[j];
        for (d = 0; d < hd; d++) {
            float o = 0.0f;
            for (j = 0; j < n; j++) o = fmaf(sc[j], V[(j0 + j) * stride + d], o);
            tile_o[t * hd + d] = o;
        }
        m[t] = mx;
        l[t] = lt;
    }
    for (t = 0; t < ntl; t++) M = fmaxf(M, m[t]);
    for (t = 0; t < ntl; t++) w[t] = or_expf(m[t] - M);
    for (t = 0; t < ntl; t++) L = fmaf(l[t], w[t], L);
    for (d = 0; d < hd; d++) {
        float O = 0.0f;
        for (t = 0; t < ntl; t++) O = fmaf(tile_o[t * hd + d], w[t], O);
        out[d] = O / L;
    }
}

int or_tile_attention(const float *qh, const float *K, const float *V, size_t stride, size_t hd,
                      size_t P, int nt, float scale, float *out)
{
    float *sc, *tile_o;
    if (!qh || !K || !V || !out || P == 0 || nt < 1 || nt > 64 || hd % 32 || hd == 0)
        return fail(OR_ERR_ARG, "tile attention: bad argument");
    sc = (float *)malloc(P * 4);
    tile_o = (float *)malloc((size_t)nt * hd * 4);
    if (!sc || !tile_o) {
        free(sc);
        free(tile_o);
        return fail(OR_ERR_ARG, "tile attention: out of memory");
    }
    tile_attention_into(qh, K, V, stride, hd, P, nt, scale, out, sc, tile_o);
    free(sc);
    free(tile_o);
    return OR_OK;
}

static void tile_attention(const or_ctx *c, const float *qh, const float *K, const float *V,
                           size_t stride, size_t hd, size_t P, float scale, float *out)
{
    tile_attention_into(qh, K, V, stride, hd, P, c->attn_nt, scale, out, c->att, c->tile_o);
}

/* one token at position c->pos; upstream forward.c:295-397 restated for a
 * single token (upstream's batched == stepped, test_forward.c:258-272) */
static int step(or_ctx *c, uint32_t token, float *hidden)
{
    const or_model *m = c->m;
    const or_model_info *mi = &m->info;
    size_t ne = mi->n_embd, hd = mi->head_dim, gqa = mi->n_head / mi->n_head_kv;
    size_t half = hd / 2, l, h, j, d, rb;
    const float *w;
    int st;
    float scale = 1.0f / sqrtf((float)hd);

    if (token >= mi->n_vocab) return fail(OR_ERR_ARG, "token outside vocabulary");
    rb = or_row_bytes(m->token_embd.type, ne);
    st = or_dequant_row(m->token_embd.type,
                        (const uint8_t *)m->token_embd.data + (size_t)token * rb, ne, c->x);
    if (st) return st;
    if (hidden) memcpy(hidden, c->x, ne * 4);

    for (l = 0; l < mi->n_layer; l++) {
        const or_layer *L = &m->layers[l];
        size_t base = l * c->n_ctx * c->nkv;
        float *kd = c->kc + base + (size_t)c->pos * c->nkv;
        float *vd = c->vc + base + (size_t)c->pos * c->nkv;
        const float *rc = c->rc + (size_t)c->pos * half, *rs = c->rs + (size_t)c->pos * half;

        if ((st = norm_w(c, &L->attn_norm, &w))) return st;
        or_rmsnorm(c->xb, c->x, w, ne, mi->rms_eps);
        if ((st = project(&L->attn_q, c->xb, c->q))) return st;
        if ((st = project(&L->attn_k, c->xb, c->k))) return st;
        if ((st = project(&L->attn_v, c->xb, c->v))) return st;
        or_rope(c->q, mi->n_head, hd, rc, rs);
        or_rope(c->k, mi->n_head_kv, hd, rc, rs);
        for (j = 0; j < c->nkv; j++) { kd[j] = kv_round(c, c->k[j]); vd[j] = kv_round(c, c->v[j]); }

        for (h = 0; h < mi->n_head; h++) {                  /* forward.c:222-257 */
            const float *qh = c->q + h * hd;
            float *dst = c->xb + h * hd;
            size_t kvh = h / gqa;
            if (c->attn_nt > 0) {
                tile_attention(c, qh, c->kc + base + kvh * hd, c->vc + base + kvh * hd, c->nkv, hd,
                               (size_t)c->pos + 1, scale, dst);
                continue;
            }
            for (j = 0; j <= c->pos; j++)
                c->att[j] = or_dot_f32(qh, c->kc + base + j * c->nkv + kvh * hd, hd) * scale;
            or_softmax(c->att, (size_t)c->pos + 1);
            for (d = 0; d < hd; d++) dst[d] = 0.0f;
            for (j = 0; j <= c->pos; j++) {
                const float *vj = c->vc + base + j * c->nkv + kvh * hd;
                float a = c->att[j];
                for (d = 0; d < hd; d++) dst[d] += a * vj[d];
            }
        }
        if ((st = project(&L->attn_out, c->xb, c->xb2))) return st;
        or_add(c->x, c->xb2, ne);

        if ((st = norm_w(c, &L->ffn_norm, &w))) return st;
        or_rmsnorm(c->xb, c->x, w, ne, mi->rms_eps);
        if ((st = project(&L->ffn_gate, c->xb, c->hb))) return st;
        if ((st = project(&L->ffn_up, c->xb, c->hb2))) return st;
        or_silu_mul(c->hb, c->hb2, mi->n_ff);
        if ((st = project(&L->ffn_down, c->hb, c->xb2))) return st;
        or_add(c->x, c->xb2, ne);
        if (hidden) memcpy(hidden + (l + 1) * ne, c->x, ne * 4);
    }
    c->pos++;
    return OR_OK;
}

int or_eval(or_ctx *c, const uint32_t *tokens, size_t n, float *logits, float *hidden)
{
    const or_model_info *mi;
    const float *w;
    size_t i;
    int st;
    if (!c || !tokens || n == 0) return fail(OR_ERR_ARG, "eval: nothing to evaluate");
    mi = &c->m->info;
    if ((size_t)c->pos + n > c->n_ctx) return fail(OR_ERR_ARG, "eval: context overrun");
    for (i = 0; i < n; i++)
        if ((st = step(c, tokens[i], i + 1 == n ? hidden : NULL))) return st;
    if (!logits) return OR_OK;
    /* forward.c:403-408: output norm and head on the last token only */
    if ((st = norm_w(c, &c->m->output_norm, &w))) return st;
    or_rmsnorm(c->xb, c->x, w, mi->n_embd, mi->rms_eps);
    return project(&c->m->output, c->xb, logits);
}

/* ---- sampler, upstream src/sample.c ----------------------------------- */

struct or_sampler {
    or_sampler_config cfg;
    size_t n_vocab, cap, len, head;
    uint64_t rng;
    float *work;
    uint32_t *hist;
};

or_sampler *or_sampler_create(const or_sampler_config *cfg, size_t n_vocab)
{
    or_sampler *s = (or_sampler *)calloc(1, sizeof(*s));
    if (!s || n_vocab == 0) { free(s); return NULL; }
    s->cfg = *cfg;                                          /* sample.c:59-66 */
    if (s->cfg.top_k < 0) s->cfg.top_k = 0;
    if (s->cfg.top_k > 512) s->cfg.top_k = 512;
    if (s->cfg.top_p <= 0.0f || s->cfg.top_p > 1.0f) s->cfg.top_p = 1.0f;
    if (s->cfg.repeat_penalty < 1.0f) s->cfg.repeat_penalty = 1.0f;
    s->n_vocab = n_vocab;
    s->rng = s->cfg.seed ? s->cfg.seed : 0x9E3779B97F4A7C15ull;
    s->cap = s->cfg.repeat_last_n ? s->cfg.repeat_last_n : 1;
    s->work = (float *)calloc(n_vocab, 4);
    s->hist = (uint32_t *)calloc(s->cap, 4);
    if (!s->work || !s->hist) { or_sampler_destroy(s); return NULL; }
    return s;
}

void or_sampler_destroy(or_sampler *s)
{
    if (!s) return;
    free(s->work); free(s->hist); free(s);
}

/* sample.c:87-93: ring of the last repeat_last_n accepted tokens */
void or_sampler_accept(or_sampler *s, uint32_t token)
{
    if (!s) return;
    s->hist[s->head] = token;
    s->head = (s->head + 1) % s->cap;
    if (s->len < s->cap) s->len++;
}

/* sample.c:32-45: xorshift64*, top 24 bits as a float in [0, 1) */
static float rng_float(uint64_t *st)
{
    uint64_t x = *st;
    x ^= x >> 12; x ^= x << 25; x ^= x >> 27;
    *st = x;
    return (float)(((x * 0x2545F4914F6CDD1Dull) >> 40) / 16777216.0);
}

typedef struct { float logit; uint32_t id; } cand;

/* sample.c:135-195 */
int or_sampler_pick(or_sampler *s, const float *logits, uint32_t *out)
{
    cand top[512];
    size_t n_top = 0, i, j;
    float mx, sum, cum, r;
    int k;
    if (!s || !logits || !out) return OR_ERR_ARG;
    memcpy(s->work, logits, s->n_vocab * 4);
    if (s->cfg.repeat_penalty > 1.0f)                        /* sample.c:95-107 */
        for (i = 0; i < s->len; i++) {
            uint32_t t = s->hist[i];
            if (t >= s->n_vocab) continue;
            if (s->work[t] > 0.0f) s->work[t] /= s->cfg.repeat_penalty;
            else s->work[t] *= s->cfg.repeat_penalty;
        }
    if (s->cfg.temperature <= 0.0f) {
        size_t best = 0;
        for (i = 1; i < s->n_vocab; i++) if (s->work[i] > s->work[best]) best = i;
        *out = (uint32_t)best;
        return OR_OK;
    }
    k = s->cfg.top_k;
    if (k <= 0 || (size_t)k > s->n_vocab) k = (int)(s->n_vocab < 512 ? s->n_vocab : 512);
    for (i = 0; i < s->n_vocab; i++) {                     /* sample.c:111-133 */
        float v = s->work[i];
        if (n_top < (size_t)k) j = n_top++;
        else { if (v <= top[n_top - 1].logit) continue; j = n_top - 1; }
        while (j > 0 && top[j - 1].logit < v) { top[j] = top[j - 1]; j--; }
        top[j].logit = v;
        top[j].id = (uint32_t)i;
    }
    mx = top[0].logit;
    sum = 0.0f;
    for (i = 0; i < n_top; i++) {
        top[i].logit = or_expf((top[i].logit - mx) / s->cfg.temperature);
        sum += top[i].logit;
    }
    if (!(sum > 0.0f)) { *out = top[0].id; return OR_OK; }
    for (i = 0; i < n_top; i++) top[i].logit /= sum;
    if (s->cfg.top_p < 1.0f) {
        cum = 0.0f;
        for (i = 0; i < n_top; i++) {
            cum += top[i].logit;
            if (cum >= s->cfg.top_p) { n_top = i + 1; break; }
        }
        sum = 0.0f;
        for (i = 0; i < n_top; i++) sum += top[i].logit;
        if (sum > 0.0f) for (i = 0; i < n_top; i++) top[i].logit /= sum;
    }
    r = rng_float(&s->rng);
    cum = 0.0f;
    for (i = 0; i < n_top; i++) {
        cum += top[i].logit;
        if (r <= cum) { *out = top[i].id; return OR_OK; }
    }
    *out = top[n_top - 1].id;
    return OR_OK;
}
