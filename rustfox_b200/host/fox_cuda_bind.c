/* libfoxcuda under RustFox's own context API, bound at link time.
 *
 * Upstream's host code (GGUF parser, weight leases, tokenizer, sampler, CLI)
 * is compiled from its sources unchanged and linked with this file and
 *   -Wl,--wrap=fox_context_create,--wrap=fox_context_destroy,
 *   --wrap=fox_context_reset,--wrap=fox_eval,--wrap=fox_context_position,
 *   --wrap=fox_context_last_eval_seconds
 * so every call from another translation unit (the CLI, an embedding
 * program) to those six entry points (include/fox/fox.h:441-450) lands here.
 * The replaced bodies are src/forward.c:56-165 (context) and :411-438
 * (fox_eval).
 *
 * fox_context_create builds upstream's context as before (its host state
 * stays valid for the rest of the API), then uploads every tensor the loader
 * resolved (src/model.c:51-83,243-252) through the weight leases to a device
 * model and creates a device context with the same position count.
 * fox_eval runs the device forward pass and hands back logits the binding
 * owns (n_vocab floats, valid until the next fox_eval on that context, as
 * upstream's are). Upstream's sampler then picks from them unchanged.
 *
 * Environment: FOX_CUDA=0 (or off) keeps upstream's CPU path; FOX_CUDA_PARITY=1
 * gives the device context fp32 K/V and upstream's serial attention order
 * (the bit-exact parity mode) instead of fp16 K/V and the tile attention. */
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "fox/fox.h"
#include "fox_internal.h"
#include "model_internal.h"
#include "foxcuda.h"

fox_status __real_fox_context_create(fox_model *m, const fox_context_config *cfg, fox_context **out);
void       __real_fox_context_destroy(fox_context *ctx);
void       __real_fox_context_reset(fox_context *ctx);
fox_status __real_fox_eval(fox_context *ctx, const uint32_t *tokens, size_t n_tokens, float **logits_out);
uint32_t   __real_fox_context_position(const fox_context *ctx);
double     __real_fox_context_last_eval_seconds(const fox_context *ctx);

/* one bound context: upstream's handle and its device counterparts */
typedef struct fox_cuda_binding {
    const fox_context       *ctx;
    foxcuda_model           *dm;
    foxcuda_context         *dc;
    float                   *logits;
    struct fox_cuda_binding *next;
} fox_cuda_binding;

static fox_cuda_binding *g_bound;
static pthread_mutex_t   g_mu = PTHREAD_MUTEX_INITIALIZER;

static int env_off(const char *name)
{
    const char *v = getenv(name);
    return v && (!strcmp(v, "0") || !strcmp(v, "off") || !strcmp(v, "no"));
}

static int env_on(const char *name)
{
    const char *v = getenv(name);
    return v && *v && !env_off(name);
}

static fox_cuda_binding *find_binding(const fox_context *ctx)
{
    fox_cuda_binding *b;
    pthread_mutex_lock(&g_mu);
    for (b = g_bound; b && b->ctx != ctx; b = b->next) {}
    pthread_mutex_unlock(&g_mu);
    return b;
}

static void free_binding(fox_cuda_binding *b)
{
    if (!b) return;
    if (b->dc) foxcuda_context_destroy(b->dc);
    if (b->dm) foxcuda_model_destroy(b->dm);
    free(b->logits);
    free(b);
}

/* one tensor through a weight lease to the device model */
static fox_status upload(fox_model *m, size_t index, int role, uint32_t layer, foxcuda_model *dm)
{
    fox_gguf_tensor t;
    fox_weights_lease lease;
    fox_status st;
    if (index == FOX_TENSOR_ABSENT) return FOX_OK; /* tied output: the device ties it too */
    st = fox_gguf_tensor_at(m->gguf, index, &t);
    if (st) return st;
    st = fox_weights_acquire(m->weights, index, &lease);
    if (st) return st;
    st = (fox_status)foxcuda_model_upload(dm, role, layer, (int)t.type, t.ne[0],
                                          t.n_dims > 1 ? t.ne[1] : 1, lease.data, (size_t)lease.bytes);
    fox_weights_release(m->weights, &lease);
    if (st) return fox_fail(st, "cuda upload: %s", foxcuda_last_error());
    return FOX_OK;
}

static fox_status attach(fox_model *m, uint32_t n_ctx, fox_cuda_binding *b)
{
    const fox_model_info *mi = &m->info;
    foxcuda_model_info info;
    foxcuda_context_config cc;
    fox_status st;
    uint32_t l;
    int r;

    info.n_layer = mi->n_layer;
    info.n_embd = mi->n_embd;
    info.n_head = mi->n_head;
    info.n_head_kv = mi->n_head_kv;
    info.n_ff = mi->n_ff;
    info.head_dim = mi->head_dim;
    info.n_vocab = mi->n_vocab;
    info.rms_eps = mi->rms_eps;
    info.rope_freq_base = mi->rope_freq_base;
    st = (fox_status)foxcuda_model_create(&info, 0, &b->dm);
    if (st) return fox_fail(st, "cuda model: %s", foxcuda_last_error());
    st = upload(m, m->token_embd, FOXCUDA_TOKEN_EMBD, 0, b->dm);
    if (!st) st = upload(m, m->output_norm, FOXCUDA_OUTPUT_NORM, 0, b->dm);
    if (!st) st = upload(m, m->output, FOXCUDA_OUTPUT, 0, b->dm);
    for (l = 0; !st && l < mi->n_layer; l++) {
        const fox_layer_tensors *L = &m->layers[l];
        const size_t index[9] = {L->attn_norm, L->attn_q, L->attn_k, L->attn_v, L->attn_out,
                                 L->ffn_norm, L->ffn_gate, L->ffn_up, L->ffn_down};
        for (r = 0; !st && r < 9; r++) st = upload(m, index[r], FOXCUDA_ATTN_NORM + r, l, b->dm);
    }
    if (st) return st;
    st = (fox_status)foxcuda_model_finalize(b->dm);
    if (st) return fox_fail(st, "cuda finalize: %s", foxcuda_last_error());
    cc.n_ctx = n_ctx;
    cc.kv_type = env_on("FOX_CUDA_PARITY") ? FOXCUDA_KV_F32 : FOXCUDA_KV_F16;
    cc.attn_exact = env_on("FOX_CUDA_PARITY") ? 1 : 0;
    st = (fox_status)foxcuda_context_create(b->dm, &cc, &b->dc);
    if (st) return fox_fail(st, "cuda context: %s", foxcuda_last_error());
    b->logits = (float *)malloc((size_t)mi->n_vocab * sizeof(float));
    if (!b->logits) return fox_fail(FOX_ERR_NOMEM, "cuda logits");
    return FOX_OK;
}

fox_status __wrap_fox_context_create(fox_model *m, const fox_context_config *cfg, fox_context **out)
{
    fox_cuda_binding *b;
    uint32_t n_ctx;
    fox_status st = __real_fox_context_create(m, cfg, out);
    if (st || env_off("FOX_CUDA")) return st;
    /* the position count upstream settles on: the config's, else the
       model's training length, else 2048 */
    n_ctx = cfg && cfg->n_ctx ? cfg->n_ctx : m->info.n_ctx_train;
    if (!n_ctx) n_ctx = 2048;
    b = (fox_cuda_binding *)calloc(1, sizeof(*b));
    if (!b) st = fox_fail(FOX_ERR_NOMEM, "cuda binding");
    if (!st) st = attach(m, n_ctx, b);
    if (st) {
        free_binding(b);
        __real_fox_context_destroy(*out);
        *out = NULL;
        return st;
    }
    b->ctx = *out;
    pthread_mutex_lock(&g_mu);
    b->next = g_bound;
    g_bound = b;
    pthread_mutex_unlock(&g_mu);
    return FOX_OK;
}

void __wrap_fox_context_destroy(fox_context *ctx)
{
    fox_cuda_binding **p, *b = NULL;
    pthread_mutex_lock(&g_mu);
    for (p = &g_bound; *p; p = &(*p)->next)
        if ((*p)->ctx == ctx) { b = *p; *p = b->next; break; }
    pthread_mutex_unlock(&g_mu);
    free_binding(b);
    __real_fox_context_destroy(ctx);
}

void __wrap_fox_context_reset(fox_context *ctx)
{
    fox_cuda_binding *b = find_binding(ctx);
    if (b) foxcuda_context_reset(b->dc);
    __real_fox_context_reset(ctx);
}

fox_status __wrap_fox_eval(fox_context *ctx, const uint32_t *tokens, size_t n_tokens, float **logits_out)
{
    fox_cuda_binding *b = find_binding(ctx);
    fox_status st;
    if (!b) return __real_fox_eval(ctx, tokens, n_tokens, logits_out);
    st = (fox_status)foxcuda_eval(b->dc, tokens, n_tokens, logits_out ? b->logits : NULL);
    if (st) return fox_fail(st, "%s", foxcuda_last_error());
    if (logits_out) *logits_out = b->logits;
    return FOX_OK;
}

uint32_t __wrap_fox_context_position(const fox_context *ctx)
{
    fox_cuda_binding *b = find_binding(ctx);
    return b ? foxcuda_context_position(b->dc) : __real_fox_context_position(ctx);
}

double __wrap_fox_context_last_eval_seconds(const fox_context *ctx)
{
    fox_cuda_binding *b = find_binding(ctx);
    return b ? foxcuda_context_last_eval_seconds(b->dc) : __real_fox_context_last_eval_seconds(ctx);
}
