/*
 * foxoracle: a plain-C restatement of RustFox's per-token forward pass.
 *
 * TEST INFRASTRUCTURE ONLY. This is the CPU checker that the parity tests,
 * the smoke check and the bench's CPU-baseline leg compare the CUDA path
 * against. The product (libfoxcuda) never links or calls it.
 *
 * Every function restates the arithmetic of the upstream C source it cites,
 * operation for operation, so that when this file and upstream are both
 * compiled with FMA contraction off their float results are identical bit for
 * bit (tests/test_oracle_vs_reference.py checks exactly that). Citations are
 * upstream paths relative to the RustFox project root.
 */
#ifndef FOXORACLE_H
#define FOXORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids, as upstream include/fox/fox.h:203-213 numbers them */
enum {
    OR_F32 = 0, OR_F16 = 1, OR_Q8_0 = 8, OR_Q4_K = 12, OR_Q6_K = 14,
    OR_TQ1_0 = 34, OR_TQ2_0 = 35
};

/* status codes, upstream include/fox/fox.h:17-26 */
enum { OR_OK = 0, OR_ERR_ARG = 1, OR_ERR_UNSUPPORTED = 5 };

/* 0 (default): exponentials through libm expf, as upstream; 1: correctly
 * rounded e^x, as the device computes it. */
void     or_set_exp_mode(int correctly_rounded);
size_t   or_expf_mismatches(uint32_t first_bits, size_t n, const float *got, size_t *first_bad);

float    or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16_rne(float f);
size_t   or_row_bytes(int type, size_t n_cols);

int  or_quantize_i8(const float *x, size_t n, int8_t *q, float *scale);
int  or_quantize_k(const float *x, size_t n, int8_t *q, float *scales);

int32_t or_tq1_block_sum(const int8_t *x, const uint8_t *block);
int32_t or_tq2_block_sum(const int8_t *x, const uint8_t *block);
/* int32 partial sums in the order upstream forms them:
 *   TQ1_0/TQ2_0: one per 256-element block                 -> rows*(n/256)
 *   Q4_K: per block, sub-blocks 0..7: dot(nibble,q), sum(q) -> rows*(n/256)*16
 *   Q6_K: per block, (half, sub) 0..3: scaled group dot      -> rows*(n/256)*4 */
int or_block_partials(int type, const int8_t *q, const void *w,
                      size_t n_rows, size_t n_cols, int32_t *out);

int or_gemv_tq_i8(int type, const int8_t *q, float act_scale, const void *w,
                  size_t n_rows, size_t n_cols, float *out);
int or_gemv(int type, const float *x, const void *w, size_t n_rows,
            size_t n_cols, float *out);
int or_dequant_row(int type, const void *row, size_t n, float *out);

void  or_rmsnorm(float *out, const float *x, const float *w, size_t n, float eps);
void  or_softmax(float *x, size_t n);
void  or_silu_mul(float *gate, const float *up, size_t n);
void  or_add(float *dst, const float *src, size_t n);
void  or_rope(float *v, size_t n_heads, size_t head_dim, const float *c, const float *s);
float or_dot_f32(const float *a, const float *b, size_t n);

typedef struct {
    uint32_t n_layer, n_embd, n_head, n_head_kv, n_ff, head_dim, n_vocab;
    float    rms_eps, rope_freq_base;
} or_model_info;

typedef struct {
    int         type;
    uint64_t    ne0, ne1;
    const void *data;
} or_tensor;

typedef struct {
    or_tensor attn_norm, attn_q, attn_k, attn_v, attn_out;
    or_tensor ffn_norm, ffn_gate, ffn_up, ffn_down;
} or_layer;

typedef struct {
    or_model_info   info;
    or_tensor       token_embd, output_norm, output;
    const or_layer *layers;
} or_model;

typedef struct or_ctx or_ctx;

/* kv_mode 0: fp32 cache exactly as upstream; 1: K and V rounded to fp16
 * (round-to-nearest-even) when written, the layout the CUDA path uses. */
or_ctx  *or_ctx_create(const or_model *m, uint32_t n_ctx, int kv_mode);
void     or_ctx_destroy(or_ctx *c);
void     or_ctx_reset(or_ctx *c);
/* 0: upstream's serial attention (the default); nt > 0: libfoxcuda's tile
 * attention with tile target nt (its production mode) */
int      or_ctx_set_attn_tiles(or_ctx *c, int nt);
/* the same tile attention for one query head over P positions of one KV
 * head (K, V rows `stride` floats apart) */
int      or_tile_attention(const float *qh, const float *K, const float *V, size_t stride,
                           size_t hd, size_t P, int nt, float scale, float *out);
uint32_t or_ctx_pos(const or_ctx *c);
/* Evaluates n tokens; logits (n_vocab) of the last token when want_logits.
 * hidden, when not NULL, receives the residual stream of the LAST token after
 * the embedding and after each layer: (n_layer + 1) * n_embd floats. */
int or_eval(or_ctx *c, const uint32_t *tokens, size_t n, float *logits,
            float *hidden);
const char *or_last_error(void);

typedef struct {
    float    temperature;
    int      top_k;
    float    top_p;
    float    repeat_penalty;
    uint32_t repeat_last_n;
    uint64_t seed;
} or_sampler_config;

typedef struct or_sampler or_sampler;
or_sampler *or_sampler_create(const or_sampler_config *cfg, size_t n_vocab);
void        or_sampler_destroy(or_sampler *s);
void        or_sampler_accept(or_sampler *s, uint32_t token);
int         or_sampler_pick(or_sampler *s, const float *logits, uint32_t *out);

#ifdef __cplusplus
}
#endif
#endif
