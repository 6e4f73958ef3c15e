/*
 * libfoxcuda -- the B200 (sm_100a) token loop behind RustFox's fox.h API.
 *
 * A C ABI of plain pointers and sizes. Every entry point returns a status with
 * the numbering of upstream's fox_status (include/fox/fox.h:17-26) and, on
 * failure, leaves a message for foxcuda_last_error() (thread-local, like
 * upstream's fox_last_error, src/log.c:40-57). Nothing aborts.
 *
 * Kernel-level entry points take DEVICE pointers and an optional CUDA stream
 * (cudaStream_t passed as void*, NULL = legacy default stream); they enqueue
 * work and return without synchronising. Model-level entry points take HOST
 * buffers and synchronise before returning, as upstream's calls do.
 *
 * Each declaration names the upstream interface it replaces (file:line in the
 * RustFox tree).
 */
#ifndef FOXCUDA_H
#define FOXCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int foxcuda_status;
enum {
    FOXCUDA_OK = 0,
    FOXCUDA_ERR_ARG,
    FOXCUDA_ERR_IO,
    FOXCUDA_ERR_NOMEM,
    FOXCUDA_ERR_FORMAT,
    FOXCUDA_ERR_UNSUPPORTED,
    FOXCUDA_ERR_NOTFOUND,
    FOXCUDA_ERR_INTERNAL
};

/* ggml type ids used here (upstream include/fox/fox.h:203-213) */
enum {
    FOXCUDA_F32 = 0, FOXCUDA_F16 = 1, FOXCUDA_Q8_0 = 8, FOXCUDA_Q4_K = 12,
    FOXCUDA_Q6_K = 14, FOXCUDA_TQ1_0 = 34, FOXCUDA_TQ2_0 = 35
};

/* replaces fox_last_error (include/fox/fox.h:30, src/log.c:40-57) */
const char *foxcuda_last_error(void);
/* replaces fox_version (include/fox/fox.h:15) */
const char *foxcuda_version(void);
/* Selects and checks the device (compute capability 10.x). */
foxcuda_status foxcuda_init(int device);

/* ---- kernel level (device pointers) ------------------------------------ */

/* replaces fox_quantize_activations_i8 (include/fox/fox.h:342-343,
 * src/gemv.c:11-42): one absmax scale for the n-vector; *scale is device. */
foxcuda_status foxcuda_quantize_activations_i8(const float *x, size_t n, int8_t *q,
                                               float *scale, void *stream);

/* The device's e^x (upstream's expf: glibc's algorithm, src/ops.c:24-48 and
 * src/sample.c:162-184 call it) of the n floats whose bit patterns are
 * first_bits, first_bits + 1, ...; out is device memory. */
foxcuda_status foxcuda_expf_range(uint32_t first_bits, size_t n, float *out, void *stream);

/* replaces fox_gemv_tq1_i8 / fox_gemv_tq2_i8 (include/fox/fox.h:350-355,
 * src/gemv.c:155-192). Weights in GGUF layout; act_scale is a device float. */
foxcuda_status foxcuda_gemv_tq1_i8(const int8_t *q, const float *act_scale,
                                   const void *weights, size_t n_rows, size_t n_cols,
                                   float *out, void *stream);
foxcuda_status foxcuda_gemv_tq2_i8(const int8_t *q, const float *act_scale,
                                   const void *weights, size_t n_rows, size_t n_cols,
                                   float *out, void *stream);

/* The per-token GEMVs of upstream's forward_batch (src/forward.c:188-213,
 * each one fox_gemv_tq{1,2}_i8, src/gemv.c:155-192) for n_tokens tokens in
 * one tensor-core pass (tcgen05 kind::i8 per 256-wide block). There is no
 * single upstream entry point.
 * - q is n_tokens x n_cols int8, token-major: each token is quantised with
 *   its own scale. act_scale holds n_tokens floats. out is n_tokens x n_rows.
 *   All are device pointers. q and the weights are 16-byte aligned.
 * - Every token's row is bit-identical to foxcuda_gemv_tq{1,2}_i8 on that
 *   token: the block sums are exact and the float fold is upstream's.
 * - foxcuda_gemm_tq_i8 takes TQ1_0 or TQ2_0 GGUF rows. It transcodes TQ1_0 to
 *   TQ2_0 (the same trits and scales) and packs into stream-ordered scratch.
 * - foxcuda_gemm_tq2_i8_packed takes TQ2_0 already packed by foxcuda_pack and
 *   allocates nothing. */
foxcuda_status foxcuda_gemm_tq_i8(int ggml_type, const int8_t *q, const float *act_scale,
                                  size_t n_tokens, const void *weights, size_t n_rows,
                                  size_t n_cols, float *out, void *stream);
foxcuda_status foxcuda_gemm_tq2_i8_packed(const int8_t *q, const float *act_scale,
                                          size_t n_tokens, const void *packed, size_t n_rows,
                                          size_t n_cols, float *out, void *stream);
/* The same for Q4_K and Q6_K weights in GGUF layout (the per-token
 * gemv_qk_i8 of src/kernels.c:571-805): q is n_tokens x n_cols int8, each
 * token quantised with one scale per 256 block (upstream
 * quantize_activations_k, src/kernels.c:722-754). act_scales holds
 * n_tokens x n_cols/256 floats. Each token's row is meant to equal the
 * single-token GEMV bit for bit. It runs 8 (Q6_K) or 16 (Q4_K) tokens per
 * tile. */
foxcuda_status foxcuda_gemm_kq_i8(int ggml_type, const int8_t *q, const float *act_scales,
                                  size_t n_tokens, const void *weights, size_t n_rows,
                                  size_t n_cols, float *out, void *stream);
/* Every tensor-core call above records a bounded wait that gave up in one
 * device error word per device (the outputs of that call are then not
 * valid). foxcuda_kernel_errors synchronises the stream, reports the word
 * and clears it. The first tensor-core call on a device looks the word up;
 * make it before any stream capture. */
foxcuda_status foxcuda_kernel_errors(void *stream);
/* The same on weights already packed by foxcuda_pack: no scratch. */
foxcuda_status foxcuda_gemm_kq_i8_packed(int ggml_type, const int8_t *q, const float *act_scales,
                                         size_t n_tokens, const void *packed, size_t n_rows,
                                         size_t n_cols, float *out, void *stream);
/* foxcuda_gemm_tq2_i8_packed with each row's blocks split over CTAs, for few
 * tokens, where the matrix alone has too few 128-row tiles to fill the GPU.
 * It writes each block's float term to terms (device scratch of
 * n_tokens x n_rows x n_cols/256 floats), then folds them in block order. The
 * result is bit-identical to the unsplit pass. */
foxcuda_status foxcuda_gemm_tq2_i8_split(const int8_t *q, const float *act_scale,
                                         size_t n_tokens, const void *packed, size_t n_rows,
                                         size_t n_cols, float *terms, float *out, void *stream);

/* replaces fox_gemv (include/fox/fox.h:363-365, src/kernels.c:809-872) for
 * TQ1_0, TQ2_0, Q4_K, Q6_K and Q8_0 weights in GGUF layout. Repacks the
 * weights into stream-ordered scratch memory, then runs the packed kernel. */
foxcuda_status foxcuda_gemv(int ggml_type, const float *x, const void *weights,
                            size_t n_rows, size_t n_cols, float *out, void *stream);

/* No counterpart in the reference: foxcuda_gemv for callers that must not
 * allocate device memory. Examples are a server whose memory is already
 * reserved for its own pool, a decode loop that must not meet an
 * out-of-memory error mid-token, and a device without stream-ordered
 * allocation. It allocates nothing. It repacks the weights into one static
 * device array of FOXCUDA_GEMV_NOALLOC_MAX_BYTES, part of the library's
 * module image, then runs the same packed kernel as foxcuda_gemv, so the
 * results are identical. A matrix whose repacked size (n_rows x row bytes)
 * exceeds the array is rejected with FOXCUDA_ERR_ARG.
 * - The first call on each device looks up the array's address with that
 *   device current. Make it before any stream capture.
 * - No part of the array has to start zeroed: each call writes every byte it
 *   reads.
 * - The array is shared. Calls that overlap in time (other streams, or
 *   unordered host threads) overwrite each other's data, so callers must
 *   order them, for instance on one stream. */
#define FOXCUDA_GEMV_NOALLOC_MAX_BYTES (32u << 20)
foxcuda_status foxcuda_gemv_noalloc(int ggml_type, const float *x, const void *weights,
                                    size_t n_rows, size_t n_cols, float *out, void *stream);

/* replaces fox_dequant_row (include/fox/fox.h:367-368, src/kernels.c:874-941)
 * for F32, F16, Q8_0, Q4_K and Q6_K. */
foxcuda_status foxcuda_dequant_row(int ggml_type, const void *row, size_t n, float *out,
                                   void *stream);

/* replaces attention_heads (src/forward.c:222-257, src/ops.c:24-39,75-81) for
 * one token: q [n_head*head_dim] (already roped), kcache / vcache
 * [n_head_kv][n_ctx][head_dim] of FOXCUDA_KV_F16 or FOXCUDA_KV_F32, positions
 * 0..pos, out [n_head*head_dim]. exact = 1 runs upstream's serial operation
 * order (bit-exact given the same exponential); 0 runs the tile attention of
 * the decode step, with the tile target foxcuda_attn_tile_target gives for
 * the current device and n_head_kv. Device pointers; scratch is
 * stream-ordered. */
/* The tile target of the tile attention (no upstream counterpart; upstream
 * attends serially, src/forward.c:222-257): the positions 0..P-1 are cut into
 * tiles of T = ceil(P / nt) and merged in tile order; nt is at most 8. A model
 * uses the value for its device and its whole model's KV heads on every
 * path (decode step, prompt chunks, batches, tensor-parallel shards). */
int foxcuda_attn_tile_target(int device, uint32_t n_head_kv);
foxcuda_status foxcuda_attention(const float *q, const void *kcache, const void *vcache,
                                 int kv_type, uint32_t n_head, uint32_t n_head_kv,
                                 uint32_t head_dim, uint32_t n_ctx, uint32_t pos, int exact,
                                 float *out, void *stream);

/* Integer partial sums exactly as upstream forms them, for bit-exact checks
 * (no single upstream entry point; the sums inside src/ternary.c:158-173,
 * 253-287 and src/kernels.c:465-569):
 *   TQ1_0/TQ2_0  n_rows*(n_cols/256)      block sums of q . (trit)
 *   Q4_K         n_rows*(n_cols/256)*16   per sub-block: dot(nibble, q), sum(q)
 *   Q6_K         n_rows*(n_cols/256)*4    per (half, sub) scaled group dot
 * q is the int8 activation vector (per-vector or per-256 quantised). */
foxcuda_status foxcuda_block_partials(int ggml_type, const int8_t *q, const void *weights,
                                      size_t n_rows, size_t n_cols, int32_t *out,
                                      void *stream);

/* The HBM weight layout: GGUF blocks regrouped into 16-byte planes per unit
 * of rows (a byte permutation). */
size_t         foxcuda_packed_bytes(int ggml_type, size_t n_rows, size_t n_cols);
foxcuda_status foxcuda_pack(int ggml_type, const void *gguf_rows, size_t n_rows,
                            size_t n_cols, void *packed, void *stream);
/* fox_gemv on already packed weights: no scratch memory. */
foxcuda_status foxcuda_gemv_packed(int ggml_type, const float *x, const void *packed,
                                   size_t n_rows, size_t n_cols, float *out, void *stream);

/* ---- model level (host buffers) ---------------------------------------- */

typedef struct foxcuda_model   foxcuda_model;
typedef struct foxcuda_context foxcuda_context;
typedef struct foxcuda_sampler foxcuda_sampler;

/* the shape fields of upstream fox_model_info (include/fox/fox.h:404-419) */
typedef struct {
    uint32_t n_layer, n_embd, n_head, n_head_kv, n_ff, head_dim, n_vocab;
    float    rms_eps, rope_freq_base;
} foxcuda_model_info;

/* tensor roles: the tensors upstream's loader resolves (src/model.c:51-83,
 * 243-252) */
enum {
    FOXCUDA_TOKEN_EMBD = 0, FOXCUDA_OUTPUT_NORM, FOXCUDA_OUTPUT,
    FOXCUDA_ATTN_NORM, FOXCUDA_ATTN_Q, FOXCUDA_ATTN_K, FOXCUDA_ATTN_V,
    FOXCUDA_ATTN_OUT, FOXCUDA_FFN_NORM, FOXCUDA_FFN_GATE, FOXCUDA_FFN_UP,
    FOXCUDA_FFN_DOWN, FOXCUDA_N_ROLES
};

/* replaces fox_model_open (include/fox/fox.h:425-426, src/model.c:146-303):
 * the caller parses GGUF and hands every tensor over with
 * foxcuda_model_upload; OUTPUT may be omitted (tied to TOKEN_EMBD,
 * src/model.c:248-252). Weights stay resident in HBM. */
foxcuda_status foxcuda_model_create(const foxcuda_model_info *info, int device,
                                    foxcuda_model **out);
foxcuda_status foxcuda_model_upload(foxcuda_model *m, int role, uint32_t layer,
                                    int ggml_type, uint64_t ne0, uint64_t ne1,
                                    const void *host_data, size_t bytes);
/* No upstream counterpart (benchmark fixtures): foxcuda_model_upload with
 * the tensor generated on the device from (seed, sigma), for synthetic
 * models too large to generate on the host quickly. Every byte is a fixed
 * function of (seed, block, field): uniform ternary weights (TQ1_0, TQ2_0)
 * or uniform bytes (Q4_K, Q6_K) with fp16 block scales |N(0, sigma)|, or
 * Q8_0 of N(0, sigma) values. Other types answer FOXCUDA_ERR_UNSUPPORTED. */
foxcuda_status foxcuda_model_upload_synthetic(foxcuda_model *m, int role, uint32_t layer,
                                              int ggml_type, uint64_t ne0, uint64_t ne1,
                                              uint64_t seed, float sigma);
foxcuda_status foxcuda_model_finalize(foxcuda_model *m);
void           foxcuda_model_destroy(foxcuda_model *m);
uint64_t       foxcuda_model_device_bytes(const foxcuda_model *m);
/* replaces fox_model_get_info (include/fox/fox.h:429): the whole model's
 * shape fields */
foxcuda_status foxcuda_model_get_info(const foxcuda_model *m, foxcuda_model_info *out);

/* Device images: the device-side counterpart of upstream's repacker
 * (fox_repack_gguf, include/fox/fox.h:262, src/repack.c:170-315), which
 * makes each layer one contiguous span of the file. An image holds a
 * finalized model (or tensor-parallel shard) exactly as it sits in HBM:
 * packed layouts, TQ1_0 layers already held as TQ2_0, norms as floats.
 * - foxcuda_model_save_image writes it (FOXCUDA_ERR_IO on a file error).
 * - foxcuda_model_open_image checks the header and every entry against the
 *   model it describes before touching the device (FOXCUDA_ERR_FORMAT),
 *   then reads the file through two pinned buffers into one device
 *   allocation: no packing kernel and no GGUF parse. An image whose
 *   matrices were laid out for another SM count is refused
 *   (FOXCUDA_ERR_UNSUPPORTED); build that model from its GGUF instead.
 * The opened model decodes exactly as the one that was saved. */
foxcuda_status foxcuda_model_save_image(const foxcuda_model *m, const char *path);
foxcuda_status foxcuda_model_open_image(const char *path, int device, foxcuda_model **out);

/* KV cache element type */
enum { FOXCUDA_KV_F16 = 0, FOXCUDA_KV_F32 = 1 };

typedef struct {
    uint32_t n_ctx;      /* positions held per sequence */
    int      kv_type;    /* FOXCUDA_KV_F16 (default) or FOXCUDA_KV_F32 */
    int      attn_exact; /* 1: attention in upstream's serial operation order
                            (bit-exact parity mode, slow); 0: split-K decode */
} foxcuda_context_config;

/* replaces fox_context_create / destroy / reset / position /
 * last_eval_seconds (include/fox/fox.h:433-450, src/forward.c:56-165) */
foxcuda_status foxcuda_context_create(foxcuda_model *m, const foxcuda_context_config *cfg,
                                      foxcuda_context **out);
/* Paged K/V cache (upstream keeps one contiguous fp32 cache per context,
 * src/forward.c:91-92). A pool holds n_pages pages per layer, each
 * FOXCUDA_KV_PAGE positions of every KV head, and is shared by contexts of
 * one model and cache type. A paged context takes ceil(n_ctx / page) pages
 * at creation (FOXCUDA_ERR_NOMEM when the pool is short) and gives them back
 * when destroyed; a block table in device memory maps its positions to
 * them, and every kernel that reads or writes K/V goes through it. Values
 * are the contiguous cache's, bit for bit. A batch takes contexts that are
 * all contiguous or all from one pool. The pool outlives its contexts:
 * foxcuda_kv_pool_destroy answers FOXCUDA_ERR_ARG while any holds pages. */
#define FOXCUDA_KV_PAGE 64
typedef struct foxcuda_kv_pool foxcuda_kv_pool;
foxcuda_status foxcuda_kv_pool_create(foxcuda_model *m, uint32_t n_pages, int kv_type,
                                      foxcuda_kv_pool **out);
uint32_t       foxcuda_kv_pool_free_pages(foxcuda_kv_pool *p);
foxcuda_status foxcuda_kv_pool_destroy(foxcuda_kv_pool *p);
foxcuda_status foxcuda_context_create_paged(foxcuda_model *m, const foxcuda_context_config *cfg,
                                            foxcuda_kv_pool *pool, foxcuda_context **out);
void           foxcuda_context_destroy(foxcuda_context *c);
void           foxcuda_context_reset(foxcuda_context *c);
uint32_t       foxcuda_context_position(const foxcuda_context *c);
double         foxcuda_context_last_eval_seconds(const foxcuda_context *c);

/* replaces fox_eval (include/fox/fox.h:446-447, src/forward.c:411-438):
 * evaluates n tokens from host memory; when logits_out is not NULL the last
 * token's n_vocab logits are copied to it (host). */
foxcuda_status foxcuda_eval(foxcuda_context *c, const uint32_t *tokens, size_t n,
                            float *logits_out);

/* Residual stream of the last evaluated token after layer `layer` (0 = the
 * embedding, n_layer = after the last layer), n_embd floats to host. Valid
 * after foxcuda_eval with foxcuda_context_set_trace(c, 1). */
foxcuda_status foxcuda_context_set_trace(foxcuda_context *c, int on);

/* How foxcuda_eval runs a prompt of several tokens (upstream forward_batch
 * over n_batch chunks, src/forward.c:295-409,411-438). No upstream
 * counterpart: upstream has one path.
 * - mode 0 (the default) runs one decode step per token.
 * - mode 1 runs chunks of up to 64 tokens. The projections take one
 *   tensor-core pass each (the kernel of foxcuda_gemm_tq_i8). RMSNorm,
 *   quantisation, RoPE, the K/V write, SwiGLU and the residual run row-wise
 *   with the decode step's arithmetic, and attention runs per token at the
 *   token's own position. Every token's values are meant to equal the
 *   step-by-step ones.
 * Mode 1 applies only to single-GPU models whose layer matrices are all
 * ternary (held as TQ2_0). Other models, trace mode and tensor-parallel
 * shards always step. */
foxcuda_status foxcuda_context_set_prefill(foxcuda_context *c, int mode);

/* fox_eval with the logits of every token: logits_out is host n x n_vocab.
 * This is the verification pass of speculative decoding, which upstream
 * plans (README.md:86-89) but does not expose: its forward_batch keeps only
 * the last row (src/forward.c:405-408).
 * - Ternary single-GPU models run in chunks, one tensor-core pass per
 *   projection, with the head on every row. Other models step.
 * - Each row equals the logits the token-by-token decode gives that token.
 * - The context advances by n. A caller that rejects part of the draft
 *   rewinds with foxcuda_context_reset and a fresh eval, as upstream has no
 *   partial rewind. */
foxcuda_status foxcuda_eval_all(foxcuda_context *c, const uint32_t *tokens, size_t n,
                                float *logits_out);
/* Back to an earlier position (no upstream counterpart; upstream only
 * resets). The cache entries from pos on are overwritten by the next
 * tokens, which is how a rejected draft is dropped. A context whose
 * tensor-parallel exchanges run over peer memory refuses it (FOXCUDA_ERR_ARG):
 * its exchange slots are tagged by position, so a replayed position would
 * read a peer's stale slot. */
foxcuda_status foxcuda_context_rewind(foxcuda_context *c, uint32_t pos);
foxcuda_status foxcuda_context_hidden(const foxcuda_context *c, uint32_t layer, float *out);

/* replaces fox_sampler_config (include/fox/fox.h:453-460) */
typedef struct {
    float    temperature;
    int      top_k;
    float    top_p;
    float    repeat_penalty;
    uint32_t repeat_last_n;
    uint64_t seed;
} foxcuda_sampler_config;

/* replaces fox_sampler_create / destroy / accept / pick (include/fox/fox.h:
 * 462-469, src/sample.c:47-195), on the device: pick reads the context's
 * current logits (the last foxcuda_eval). repeat_last_n <= 1024. */
foxcuda_status foxcuda_sampler_create(foxcuda_context *c, const foxcuda_sampler_config *cfg,
                                      foxcuda_sampler **out);
void           foxcuda_sampler_destroy(foxcuda_sampler *s);
foxcuda_status foxcuda_sampler_accept(foxcuda_sampler *s, uint32_t token);
foxcuda_status foxcuda_sampler_pick(foxcuda_sampler *s, uint32_t *out);

/* One decode step of upstream's `fox run` loop (src/cli.c:340-361) as one
 * CUDA graph: eval `token`, pick the next token, accept it into the sampler
 * history; the pick is returned in *next (host). */
foxcuda_status foxcuda_decode(foxcuda_context *c, foxcuda_sampler *s, uint32_t token,
                              uint32_t *next);

/* n decode steps with the picked token fed back on the device (no host round
 * trip between steps); out receives the n picks (host). */
foxcuda_status foxcuda_generate(foxcuda_context *c, foxcuda_sampler *s, uint32_t token,
                                size_t n, uint32_t *out);

/* ---- decode batches (no upstream counterpart: upstream decodes one
 * sequence per context, src/forward.c:411-438) ----------------------------
 * A batch is a set of contexts of one single-GPU ternary model (layer
 * matrices held as TQ2_0), equal in length, cache type and attention mode. A
 * batch step advances every context by one token in one pass: the row
 * kernels and one tensor-core pass per projection serve all of them, and
 * each context keeps its own cache, position, logits and sampler. Every
 * context's values are meant to equal its own decode step's, bit for bit.
 * At most 64 contexts per batch. */
typedef struct foxcuda_batch foxcuda_batch;
foxcuda_status foxcuda_batch_create(foxcuda_context *const *ctxs, size_t n, foxcuda_batch **out);
void           foxcuda_batch_destroy(foxcuda_batch *b);
/* One token per context: tokens (host, n ids) or NULL for each context's
 * device token (its last pick). logits: NULL or host n x n_vocab. */
foxcuda_status foxcuda_batch_step(foxcuda_batch *b, const uint32_t *tokens, float *logits);
/* n_steps steps, each followed by a pick with samplers[i] for context i and
 * the picks fed back on the device (one CUDA graph per step). first: the
 * first tokens (host, n ids) or NULL for the device tokens. out: host,
 * n_steps x n, step-major. */
foxcuda_status foxcuda_batch_generate(foxcuda_batch *b, foxcuda_sampler *const *samplers,
                                      const uint32_t *first, size_t n_steps, uint32_t *out);
double         foxcuda_batch_last_seconds(const foxcuda_batch *b);
/* One batch step on host tokens with a CUDA event after each phase (embed,
 * then per layer qkv, attention, o, gate_up, down, then head, advance): the
 * phase kinds (as foxcuda_context_profile numbers them) and microseconds,
 * at most cap of them, their count in *n_out. */
foxcuda_status foxcuda_batch_profile(foxcuda_batch *b, const uint32_t *tokens, float *us, int *kinds,
                                     int cap, int *n_out);
/* Benchmark stand-in for a long prompt: positions [0, n_pos) of every layer's
 * K and V are set to seeded N(0, 1) values and the position to n_pos. */
foxcuda_status foxcuda_context_fill_kv(foxcuda_context *c, uint32_t n_pos, uint64_t seed);

/* ---- tensor parallel (no upstream counterpart: upstream runs one process,
 * src/threadpool.c; the split follows the scheme of include/fox/fox.h's
 * fox_eval with Megatron-style shards) ------------------------------------
 * Shard tp_rank of tp_size: q/k/v rows by heads, gate/up rows by 256-wide FFN
 * blocks, head rows by vocabulary range (column-parallel); attn_output and
 * ffn_down by the matching column blocks (row-parallel). A row-parallel shard
 * quantises with the absmax of the whole vector (a max over shards), emits
 * its per-block float terms, and every shard folds the gathered terms in
 * upstream's block order: the sharded decode equals the unsharded one bit for
 * bit. The steps below only enqueue work on foxcuda_context_stream(); the
 * caller puts its collectives (max-allreduce of one float, all-gathers of the
 * terms and of the {value, index} pairs) on the same stream between them. */
typedef struct {
    int32_t  tp_rank, tp_size;
    uint32_t n_head, n_head_kv, n_ff;   /* this shard's heads and FFN width */
    uint32_t vocab_begin, n_vocab;      /* this shard's head rows */
    uint32_t o_blocks;                  /* attn_output column blocks per shard */
    uint32_t ffn_blocks[8];             /* ffn_down column blocks of every shard */
    uint32_t o_terms, down_terms;       /* float terms per block (1 ternary, 8 Q4_K,
                                           4 Q6_K), the most over the layers */
} foxcuda_tp_shape;

foxcuda_status foxcuda_model_create_tp(const foxcuda_model_info *info, int device, int tp_rank,
                                       int tp_size, foxcuda_model **out);
foxcuda_status foxcuda_tp_info(const foxcuda_model *m, foxcuda_tp_shape *out);
void          *foxcuda_context_stream(foxcuda_context *c);
/* token >= 0 comes from the host; token < 0 embeds the last foxcuda_tp_pick */
foxcuda_status foxcuda_tp_embed(foxcuda_context *c, int64_t token);
foxcuda_status foxcuda_tp_attention(foxcuda_context *c, uint32_t layer);
/* which: 0 = attention output (o input), 1 = FFN hidden (down input); device float */
foxcuda_status foxcuda_tp_amax(foxcuda_context *c, int which, float *amax);
foxcuda_status foxcuda_tp_terms(foxcuda_context *c, uint32_t layer, int which,
                                const float *amax_all, float *terms, uint32_t stride);
foxcuda_status foxcuda_tp_fold(foxcuda_context *c, uint32_t layer, int which,
                               const float *gathered, uint32_t stride, const float *amax_all);
foxcuda_status foxcuda_tp_ffn(foxcuda_context *c, uint32_t layer);
/* best = {value, index bits} (2 device floats) */
foxcuda_status foxcuda_tp_head(foxcuda_context *c, float *best);
/* pairs = tp_size gathered {value, index} pairs (device); pos += 1 */
foxcuda_status foxcuda_tp_pick(foxcuda_context *c, const float *pairs);
foxcuda_status foxcuda_tp_advance(foxcuda_context *c);
/* the next step's token copied from pinned host memory into the device word
 * foxcuda_tp_embed(c, -1) reads (for a captured step fed from the host) */
foxcuda_status foxcuda_tp_feed(foxcuda_context *c, uint32_t token);
foxcuda_status foxcuda_tp_tokens(foxcuda_context *c, uint32_t first_pos, size_t n, uint32_t *out);
/* the host's position counter re-read from the device (after replaying a
 * captured foxcuda_tp_* step, which advances only the device's) */
foxcuda_status foxcuda_context_sync_position(foxcuda_context *c);
/* this shard's logits of its last head evaluation (n <= its vocabulary rows) */
foxcuda_status foxcuda_context_logits(foxcuda_context *c, float *out, size_t n);

/* The same exchanges over peer memory (NVLink) instead of host collectives.
 * Each rank's context owns an exchange arena. The arena holds every rank's
 * absmax and pick slots, readiness flags, and this rank's block terms, and
 * it is shared through CUDA IPC (plain peer loads and stores only).
 * - foxcuda_tp_p2p_export writes this arena's IPC handle
 *   (FOXCUDA_IPC_HANDLE_BYTES).
 * - After every rank has exported, foxcuda_tp_p2p_open maps the others'
 *   arenas. handles holds world x FOXCUDA_IPC_HANDLE_BYTES, rank order.
 * - foxcuda_tp_p2p_row replaces amax + max-allreduce + terms + all-gather +
 *   fold of one row-parallel projection. foxcuda_tp_p2p_pick replaces
 *   head + all-gather + pick.
 * - Two exchanges (foxcuda_tp_p2p_mode, the same on every rank, set
 *   between steps):
 *   FOXCUDA_TP_TERMS (default)  two kernels: the terms GEMV with the absmax
 *     exchange and the readiness signal inside it, then the fold of every
 *     rank's block terms in upstream's order. The values and their order are those of
 *     the collective form: the single-GPU decode's, bit for bit.
 *   FOXCUDA_TP_SUMS  one kernel: the GEMV trades the absmax, folds this
 *     shard's blocks per row and pushes the n_embd row values (rank 0's
 *     with the residual added) to every rank; the next GEMV over the
 *     residual (q|k|v or gate|up of this context) adds the ranks' rows in
 *     rank order in its prologue, and the head is preceded by that sum as a
 *     kernel of its own. Same result on every rank; the single-GPU decode's
 *     up to float rounding of the partial sums (one rank: bit for bit).
 * - Every wait is bounded. A wait that gives up sets the device error word
 *   (code 2), which foxcuda_tp_tokens and later calls report.
 * - After foxcuda_context_reset, and after any call that reports the error
 *   word, every rank calls foxcuda_tp_p2p_clear before any rank's next step:
 *   a step whose wait gave up leaves its terms and slots unusable. */
/* Repeat penalty of the sharded greedy pick (upstream src/sample.c:95-107):
 * each shard penalises the history tokens of its own vocabulary rows before
 * its argmax. Prompt tokens given to foxcuda_tp_embed from the host, and
 * every pick, enter the history, as `fox run` accepts them. The pick equals
 * the unsharded sampler's. Call before the first step; penalty 1 leaves the
 * pick plain greedy. */
foxcuda_status foxcuda_tp_set_penalty(foxcuda_context *c, float penalty, uint32_t last_n);

#define FOXCUDA_IPC_HANDLE_BYTES 64
foxcuda_status foxcuda_tp_p2p_export(foxcuda_context *c, void *handle);
foxcuda_status foxcuda_tp_p2p_open(foxcuda_context *c, const void *handles);
/* The peers' arenas from contexts of this process (one process driving
 * several GPUs): ranks[k] is rank k's exported context, this one at its own
 * rank. Peer access is enabled between distinct devices. Two ranks on one
 * GPU must not both step: each rank's exchange waits for kernels of the
 * other, and nothing makes two launches on one GPU run at the same time. */
foxcuda_status foxcuda_tp_p2p_open_local(foxcuda_context *c, foxcuda_context *const *ranks);
foxcuda_status foxcuda_tp_p2p_clear(foxcuda_context *c);
foxcuda_status foxcuda_tp_p2p_row(foxcuda_context *c, uint32_t layer, int which);
foxcuda_status foxcuda_tp_p2p_pick(foxcuda_context *c);
enum { FOXCUDA_TP_TERMS = 0, FOXCUDA_TP_SUMS = 1 };
foxcuda_status foxcuda_tp_p2p_mode(foxcuda_context *c, int mode);

/* ---- diagnostics (no upstream counterpart; upstream only times whole evals,
 * src/forward.c:421-435) ------------------------------------------------- */

/* Launch kinds of a decode step */
enum {
    FOXCUDA_K_EMBED = 0, FOXCUDA_K_QKV, FOXCUDA_K_ATTN, FOXCUDA_K_O, FOXCUDA_K_GATEUP,
    FOXCUDA_K_DOWN, FOXCUDA_K_ADVANCE, FOXCUDA_K_HEAD, FOXCUDA_K_PICK
};

/* One decode step of `token` (plus a pick when s is not NULL) run launch by
 * launch with an event after each, so every launch's device time is
 * separated. Writes up to cap (microseconds, kind) pairs; advances the
 * context like a decode step. */
foxcuda_status foxcuda_context_profile(foxcuda_context *c, foxcuda_sampler *s, uint32_t token,
                                       float *us, int *kinds, int cap, int *n_out);

/* Average device time of one launch of a layer GEMV kind (QKV, O, GATEUP,
 * DOWN or HEAD) over `reps` back-to-back launches on the context's stream,
 * cycling through the layers so the weights stream from HBM, and the GGUF
 * weight bytes one launch reads. Overwrites the context's activations and the
 * cache slot at the current position: reset the context before decoding. */
foxcuda_status foxcuda_context_bench_kernel(foxcuda_context *c, int kind, int reps,
                                            double *us_per_launch,
                                            uint64_t *weight_bytes_per_launch);

#ifdef __cplusplus
}
#endif
#endif
