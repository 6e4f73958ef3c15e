/* `fox run --temp 0` on token ids through upstream's public API
 * (src/cli.c:312-361 without the tokenizer): open a GGUF, create a context,
 * evaluate the prompt, accept it into upstream's sampler (temperature 0,
 * repeat penalty 1.1 over the last 64), then pick, accept and evaluate one
 * token at a time. Prints the picked ids on one line.
 *
 *   fox_cuda_ids <model.gguf> <n_ctx> <n_generate> <prompt id>...
 *
 * Linked with fox_cuda_bind.c the context and fox_eval run on the device;
 * FOX_CUDA=0 keeps upstream's CPU path in the same binary. */
#include <stdio.h>
#include <stdlib.h>

#include "fox/fox.h"

int main(int argc, char **argv)
{
    fox_model *model = NULL;
    fox_context *ctx = NULL;
    fox_sampler *smp = NULL;
    fox_context_config cc;
    fox_sampler_config sc = {0.0f, 40, 0.95f, 1.1f, 64, 0};
    uint32_t *ids = NULL, next = 0;
    float *logits = NULL;
    unsigned long n_gen, i;
    int n_prompt, k, rc = 1;

    if (argc < 5) {
        fprintf(stderr, "usage: fox_cuda_ids <model.gguf> <n_ctx> <n_generate> <prompt id>...\n");
        return 2;
    }
    n_prompt = argc - 4;
    n_gen = strtoul(argv[3], NULL, 10);
    ids = (uint32_t *)malloc((size_t)n_prompt * sizeof(uint32_t));
    if (!ids) return 1;
    for (k = 0; k < n_prompt; k++) ids[k] = (uint32_t)strtoul(argv[4 + k], NULL, 10);

    if (fox_model_open(argv[1], FOX_WEIGHTS_RESIDENT, 0, &model) != FOX_OK) goto fail;
    fox_context_config_default(&cc, model);
    cc.n_ctx = (uint32_t)strtoul(argv[2], NULL, 10);
    if (fox_context_create(model, &cc, &ctx) != FOX_OK) goto fail;
    smp = fox_sampler_create(&sc, fox_model_get_info(model)->n_vocab);
    if (!smp) goto fail;
    if (fox_eval(ctx, ids, (size_t)n_prompt, &logits) != FOX_OK) goto fail;
    for (k = 0; k < n_prompt; k++) fox_sampler_accept(smp, ids[k]);
    for (i = 0; i < n_gen; i++) {
        if (fox_sampler_pick(smp, logits, &next) != FOX_OK) goto fail;
        fox_sampler_accept(smp, next);
        printf(i ? " %u" : "%u", next);
        if (i + 1 < n_gen && fox_eval(ctx, &next, 1, &logits) != FOX_OK) goto fail;
    }
    printf("\n");
    fprintf(stderr, "position %u\n", fox_context_position(ctx));
    rc = 0;
    goto done;
fail:
    fprintf(stderr, "fox_cuda_ids: %s\n", fox_last_error());
done:
    if (smp) fox_sampler_destroy(smp);
    if (ctx) fox_context_destroy(ctx);
    if (model) fox_model_close(model);
    free(ids);
    return rc;
}
