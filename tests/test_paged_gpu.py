"""The paged K/V cache (foxcuda_kv_pool_*, foxcuda_context_create_paged)
against the contiguous cache, bit for bit.

Upstream keeps one contiguous fp32 cache per context (src/forward.c:91-92).
A paged context's positions live in pages of a shared pool, scattered in the
pool's shuffled order, and every kernel that writes or reads K/V goes
through the context's block table. Only the addresses change, so every
logit, every layer and every pick must equal the contiguous context's: in
production mode (tile attention, fp16) and parity mode (serial attention,
fp32), stepping and prompt chunks, single contexts and batches, and the
seeded long-context fill. The pool's accounting is checked too.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from rustfox_b200 import formats as F, synth  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

CFG = synth.CONFIGS["tiny"].scaled(name="tiny-paged", n_layer=3)
CFG_TQ2 = CFG.scaled(name="tiny-paged-tq2", linear_type=F.TQ2_0)
N_CTX = 200  # not a multiple of the page: the last page is partly used
PROMPT = synth.random_prompt(CFG, 70, seed=4)  # crosses a page boundary
MODELS = {}


def _model(cfg):
    if cfg.name not in MODELS:
        MODELS[cfg.name] = rf.Model.from_synthetic(synth.generate(cfg))
    return MODELS[cfg.name]


def _pages(n_ctx):
    return (n_ctx + rf.api.KV_PAGE - 1) // rf.api.KV_PAGE


@pytest.mark.parametrize("kv,exact", [("f16", False), ("f32", True)], ids=["production", "parity"])
def test_paged_context_equals_contiguous_every_layer(kv, exact):
    m = _model(CFG)
    pool = m.kv_pool(3 * _pages(N_CTX), kv=kv)
    other = rf.Context(m, N_CTX, kv=kv, attn_exact=exact, pool=pool)  # takes pages first: a gap
    a = rf.Context(m, N_CTX, kv=kv, attn_exact=exact)
    b = rf.Context(m, N_CTX, kv=kv, attn_exact=exact, pool=pool)
    for c in (a, b):
        c.set_trace(True)
    want, got = a.eval(PROMPT), b.eval(PROMPT)
    for l in range(CFG.n_layer + 1):
        assert np.array_equal(a.hidden(l).view(np.uint32), b.hidden(l).view(np.uint32)), f"layer {l}"
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))
    for t in synth.random_prompt(CFG, 40, seed=6):  # decode steps into later pages
        assert np.array_equal(a.eval([t]).view(np.uint32), b.eval([t]).view(np.uint32))
    for c in (a, b, other):
        c.close()
    pool.close()


@pytest.mark.parametrize("cfg", [CFG, CFG_TQ2], ids=["tq1", "tq2"])
def test_paged_greedy_equals_contiguous(cfg):
    m = _model(cfg)
    pool = m.kv_pool(_pages(N_CTX))
    want = rf.greedy_generate(m, PROMPT, 100, N_CTX)
    got = rf.greedy_generate(m, PROMPT, 100, N_CTX, pool=pool)
    assert np.array_equal(got, want), f"first divergence at {np.argmax(got != want)}"
    assert pool.free_pages == _pages(N_CTX)
    pool.close()


def test_paged_prompt_chunks_equal_contiguous_steps():
    """Prompt chunks through the tensor cores write K/V through the table too."""
    m = _model(CFG_TQ2)
    pool = m.kv_pool(_pages(N_CTX))
    a = rf.Context(m, N_CTX)
    b = rf.Context(m, N_CTX, pool=pool)
    b.set_prefill(True)
    want, got = a.eval(PROMPT), b.eval(PROMPT)
    assert np.array_equal(want.view(np.uint32), got.view(np.uint32))
    for t in synth.random_prompt(CFG, 8, seed=7):
        assert np.array_equal(a.eval([t]).view(np.uint32), b.eval([t]).view(np.uint32))
    a.close()
    b.close()
    pool.close()


def test_paged_batch_equals_contiguous_batch():
    m = _model(CFG_TQ2)
    pool = m.kv_pool(4 * _pages(N_CTX))
    starts = [5, 66, 130]  # positions in different pages

    def contexts(pool_or_none):
        out = []
        for i, n in enumerate(starts):
            c = rf.Context(m, N_CTX, pool=pool_or_none)
            c.eval(synth.random_prompt(CFG, n, seed=20 + i))
            out.append(c)
        return out

    toks = synth.random_prompt(CFG, 3 * len(starts), seed=8).reshape(3, len(starts))
    runs = []
    for p in (None, pool):
        ctxs = contexts(p)
        b = rf.Batch(ctxs)
        runs.append([b.step(row).view(np.uint32) for row in toks])
        b.close()
        for c in ctxs:
            c.close()
    for k in range(len(toks)):
        for i in range(len(starts)):
            assert np.array_equal(runs[0][k][i], runs[1][k][i]), f"step {k}, context {i}"
    pool.close()


def test_paged_fill_kv_equals_contiguous():
    m = _model(CFG_TQ2)
    pool = m.kv_pool(_pages(N_CTX))
    a = rf.Context(m, N_CTX)
    b = rf.Context(m, N_CTX, pool=pool)
    for c in (a, b):
        c.fill_kv(150, seed=9)
    t = [int(synth.random_prompt(CFG, 1, seed=10)[0])]
    assert np.array_equal(a.eval(t).view(np.uint32), b.eval(t).view(np.uint32))
    a.close()
    b.close()
    pool.close()


def test_pool_accounting():
    m = _model(CFG)
    per = _pages(N_CTX)
    pool = m.kv_pool(2 * per + 1)
    assert pool.free_pages == 2 * per + 1
    a = rf.Context(m, N_CTX, pool=pool)
    b = rf.Context(m, N_CTX, pool=pool)
    assert pool.free_pages == 1
    with pytest.raises(rf.FoxError) as e:
        rf.Context(m, N_CTX, pool=pool)
    assert e.value.status == rf.api.ERR_NOMEM
    with pytest.raises(rf.FoxError):
        pool.close()  # contexts still hold pages
    a.close()
    c = rf.Context(m, N_CTX, pool=pool)  # the freed pages are taken again
    assert pool.free_pages == 1
    with pytest.raises(rf.FoxError):
        rf.Context(m, N_CTX, kv="f32", pool=pool)  # the pool's cache type is f16
    b.close()
    c.close()
    assert pool.free_pages == 2 * per + 1
    pool.close()


def test_batch_refuses_mixed_paging():
    m = _model(CFG_TQ2)
    pool = m.kv_pool(_pages(N_CTX))
    a = rf.Context(m, N_CTX)
    b = rf.Context(m, N_CTX, pool=pool)
    with pytest.raises(rf.FoxError):
        rf.Batch([a, b])
    a.close()
    b.close()
    pool.close()
