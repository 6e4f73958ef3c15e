"""Prompt chunks through the tensor-core pass (foxcuda_context_set_prefill)
against the token-by-token decode, bit for bit.

Upstream's fox_eval runs a prompt through forward_batch in chunks, with one
GEMV per token and projection (src/forward.c:188-213, 295-438), so its
values are the step-by-step ones. The chunk mode here must equal the decode
step on every token. The test checks the logits after the prompt, and the
logits of further single tokens, which read the K/V the chunks wrote. The
cases cover one chunk, two chunks (64 + 36 tokens), a prompt of two tokens,
both ternary types, and both cache modes.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from rustfox_b200 import formats as F, synth  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

N_CTX = 160
TINY = synth.CONFIGS["tiny"].scaled(name="tiny-prefill", n_layer=3)
TINY_TQ2 = TINY.scaled(name="tiny-prefill-tq2", linear_type=F.TQ2_0)
MODELS = {}


def _model(cfg):
    if cfg.name not in MODELS:
        MODELS[cfg.name] = rf.Model.from_synthetic(synth.generate(cfg))
    return MODELS[cfg.name]


def _run(model, prompt, more, chunks, kv, exact):
    ctx = rf.Context(model, N_CTX, kv=kv, attn_exact=exact)
    ctx.set_prefill(chunks)
    out = [ctx.eval(prompt)]
    for t in more:
        out.append(ctx.eval([t]))
    assert ctx.pos == len(prompt) + len(more)
    ctx.close()
    return np.stack(out).view(np.uint32)


@pytest.mark.parametrize("cfg", [TINY, TINY_TQ2], ids=["tq1", "tq2"])
@pytest.mark.parametrize("kv,exact", [("f16", False), ("f32", True)], ids=["production", "parity"])
@pytest.mark.parametrize("n_prompt", [2, 40, 100])
def test_chunks_equal_steps(cfg, kv, exact, n_prompt):
    model = _model(cfg)
    prompt = synth.random_prompt(cfg, n_prompt, seed=n_prompt)
    more = synth.random_prompt(cfg, 3, seed=99)
    steps = _run(model, prompt, more, False, kv, exact)
    chunks = _run(model, prompt, more, True, kv, exact)
    bad = np.argwhere(steps != chunks)
    assert bad.size == 0, f"{len(bad)} logits differ, first at (eval, index) {tuple(bad[0])}"


def test_set_prefill_rejects_unknown_modes():
    ctx = rf.Context(_model(TINY), 16)
    assert rf.lib().foxcuda_context_set_prefill(ctx.h, 2) == 1 and rf.last_error()
    ctx.close()
