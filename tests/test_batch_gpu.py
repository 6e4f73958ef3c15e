"""Decode batches (foxcuda_batch_*) against each context's own decode step,
bit for bit.

Upstream decodes one sequence per context (src/forward.c:411-438). A batch
step serves several contexts with one pass; every context's logits and
picks must equal what its own decode step gives. The cases cover contexts at
different positions, both ternary types, both cache modes, greedy and
seeded top-k sampling, and the synthetic long-context fill.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from rustfox_b200 import formats as F, synth  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

N_CTX = 96
TINY = synth.CONFIGS["tiny"].scaled(name="tiny-batch", n_layer=3)
TINY_TQ2 = TINY.scaled(name="tiny-batch-tq2", linear_type=F.TQ2_0)
# config 5's kind: ternary layers with a Q6_K head (one K-quant pass for all heads)
TINY_Q6H = TINY.scaled(name="tiny-batch-q6h", linear_type=F.TQ2_0, output_type=F.Q6_K)
MODELS = {}
PROMPTS = [5, 17, 30]


def _model(cfg):
    if cfg.name not in MODELS:
        MODELS[cfg.name] = rf.Model.from_synthetic(synth.generate(cfg))
    return MODELS[cfg.name]


def _contexts(model, cfg, kv, exact):
    out = []
    for i, n in enumerate(PROMPTS):
        c = rf.Context(model, N_CTX, kv=kv, attn_exact=exact)
        c.eval(synth.random_prompt(cfg, n, seed=10 + i))
        out.append(c)
    return out


@pytest.mark.parametrize("cfg", [TINY, TINY_TQ2, TINY_Q6H], ids=["tq1", "tq2", "tq2-q6k-head"])
@pytest.mark.parametrize("kv,exact", [("f16", False), ("f32", True)], ids=["production", "parity"])
def test_batch_steps_equal_single_steps(cfg, kv, exact):
    model = _model(cfg)
    toks = synth.random_prompt(cfg, 4 * len(PROMPTS), seed=3).reshape(4, len(PROMPTS))
    solo = _contexts(model, cfg, kv, exact)
    want = [[c.eval([t]).view(np.uint32) for c, t in zip(solo, row)] for row in toks]
    ctxs = _contexts(model, cfg, kv, exact)
    b = rf.Batch(ctxs)
    got = [b.step(row).view(np.uint32) for row in toks]
    for k in range(len(toks)):
        for i in range(len(PROMPTS)):
            bad = np.count_nonzero(got[k][i] != want[k][i])
            assert bad == 0, f"step {k}, context {i}: {bad} logits differ"
    assert [c.pos for c in ctxs] == [c.pos for c in solo]
    b.close()
    for c in solo + ctxs:
        c.close()


@pytest.mark.parametrize("temperature", [0.0, 0.8], ids=["greedy", "top-k"])
def test_batch_generate_equals_generate(temperature):
    cfg = TINY_TQ2
    model = _model(cfg)
    first = synth.random_prompt(cfg, len(PROMPTS), seed=4)
    kw = dict(temperature=temperature, top_k=40, top_p=1.0, repeat_penalty=1.0)
    solo = _contexts(model, cfg, "f16", False)
    want = np.stack([rf.Sampler(c, seed=7 + i, **kw).generate(int(t), 12)
                     for i, (c, t) in enumerate(zip(solo, first))], axis=1)
    ctxs = _contexts(model, cfg, "f16", False)
    smp = [rf.Sampler(c, seed=7 + i, **kw) for i, c in enumerate(ctxs)]
    b = rf.Batch(ctxs)
    got = np.concatenate([b.generate(smp, 5, first=first), b.generate(smp, 7)])
    assert np.array_equal(got, want)
    b.close()


def test_fill_kv_is_seeded():
    model = _model(TINY_TQ2)
    lg = []
    for _ in range(2):
        c = rf.Context(model, N_CTX)
        c.fill_kv(80, seed=3)
        assert c.pos == 80
        lg.append(c.eval([5]).view(np.uint32))
        c.close()
    assert np.array_equal(lg[0], lg[1])


def test_batch_rejects_mixed_contexts():
    model = _model(TINY_TQ2)
    a, b = rf.Context(model, 32), rf.Context(model, 48)
    with pytest.raises(rf.FoxError):
        rf.Batch([a, b])
    with pytest.raises(rf.FoxError):
        rf.Batch([a, a])
    a.close()
    b.close()
