"""The decode step at the benchmark shapes against the CPU oracle, bit for bit.

The other end-to-end tests run the tiny shape. The kernels' geometry (units
per CTA, row slots per block column, clusters per KV head, the head's row
units) depends on the matrix shapes and the SM count, so the benchmarked
shapes get their own check here:
  4b    config 2 (hidden 2560, 32/8 heads of 128, FFN 9728, vocab 151936,
        TQ1_0 layers held as TQ2_0, Q8_0 embedding and head), 2 layers;
  27b   config 4's layer shapes (hidden 5120, 32/16 heads, FFN 21504, TQ2_0),
        1 layer, with a 32000-entry vocabulary so the host can build it.
Both attention modes are held bit for bit against the oracle: parity mode
(fp32 cache, upstream's serial attention) and production mode (fp16 cache,
the tile attention the oracle restates), at every layer and on the logits,
and greedy decoding picks the same tokens (upstream src/forward.c:295-409,
src/gemv.c:54-97).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
from rustfox_b200 import synth  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

from conftest import rel_l2  # noqa: E402

SHAPES = {
    "4b": synth.CONFIGS["4b"].scaled(name="4b-2", n_layer=2),
    "27b": synth.CONFIGS["27b"].scaled(name="27b-1", n_layer=1, n_vocab=32000),
}
N_CTX = 96


@pytest.fixture(scope="module", params=sorted(SHAPES))
def shape(request):
    cfg = SHAPES[request.param]
    host = synth.generate(cfg)
    m = rf.Model.from_synthetic(host)
    yield cfg, m, O.OracleModel(host)
    m.close()


def _modes(m):
    return {"parity": dict(kv="f32", attn_exact=True, oracle=dict(kv_fp16=False, attn_tiles=0)),
            "production": dict(kv="f16", attn_exact=False,
                               oracle=dict(kv_fp16=True, attn_tiles=m.attn_tiles))}


@pytest.mark.parametrize("mode", ["parity", "production"])
def test_every_layer_and_the_logits_bit_identical(shape, mode):
    cfg, m, om = shape
    md = _modes(m)[mode]
    prompt = synth.random_prompt(cfg, 24, seed=7)
    want, want_h = om.context(N_CTX, **md["oracle"]).eval(prompt, want_hidden=True)
    ctx = m.context(N_CTX, kv=md["kv"], attn_exact=md["attn_exact"])
    ctx.set_trace(True)
    got = ctx.eval(prompt)
    for l in range(cfg.n_layer + 1):
        h = ctx.hidden(l)
        assert np.array_equal(h.view(np.uint32), want_h[l].view(np.uint32)), (
            f"{cfg.name} {mode} layer {l}: rel L2 {rel_l2(h, want_h[l]):.3g}")
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (
        f"{cfg.name} {mode} logits: rel L2 {rel_l2(got, want):.3g}")
    ctx.close()


@pytest.mark.parametrize("mode", ["parity", "production"])
def test_greedy_tokens_identical(shape, mode):
    cfg, m, om = shape
    md = _modes(m)[mode]
    prompt = synth.random_prompt(cfg, 16, seed=8)
    n_gen = 32 if cfg.name.startswith("4b") else 16
    want = O.greedy_generate(om, prompt, n_gen, N_CTX, **md["oracle"])
    got = rf.greedy_generate(m, prompt, n_gen, N_CTX, kv=md["kv"], attn_exact=md["attn_exact"])
    assert np.array_equal(got, want), f"{cfg.name} {mode}: first divergence at {np.argmax(got != want)}"


def test_step_is_one_launch_per_kernel_kind(shape):
    """At these shapes the decode step is embed, then per layer qkv,
    attention, o, gate_up, down, then the position advance and the head:
    no split, no extra reduction launch."""
    cfg, m, _ = shape
    ctx = m.context(N_CTX)
    ctx.eval(synth.random_prompt(cfg, 4, seed=9), want_logits=False)
    kinds = [k for k, _ in ctx.profile_step(5)]
    layer = ["qkv", "attention", "o", "gate_up", "down"]
    assert kinds == ["embed"] + layer * cfg.n_layer + ["advance", "head"], kinds
    ctx.close()
