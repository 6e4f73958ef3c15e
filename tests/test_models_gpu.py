"""The other weight formats of the benchmark configs, end to end on the device.

Config 3 (8B) uses Q4_K for the linear weights with Q6_K attn_v and head;
configs 4 and 5 use TQ2_0 linear weights. They run here at the tiny shape,
with the same formats, seeded the same way: parity mode (fp32 cache, upstream's
attention order) and production mode (fp16 cache, the tile attention, which
the oracle restates) must reproduce the oracle bit for bit at every layer,
and greedy decoding must pick the same tokens. The K-quant layers and the
Q6_K head go through the ring-mode unit GEMV, the TQ2_0 layers through the
persistent decode step without transcoding.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
from rustfox_b200 import formats as F, synth  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

from conftest import rel_l2  # noqa: E402

TINY = synth.CONFIGS["tiny"]
VARIANTS = {
    "q4k": TINY.scaled(name="tiny-q4k", n_layer=4, linear_type=F.Q4_K, attn_v_type=F.Q6_K,
                       output_type=F.Q6_K, linear_sigma=0.01),
    "tq2": TINY.scaled(name="tiny-tq2", n_layer=4, linear_type=F.TQ2_0),
}


@pytest.fixture(scope="module", params=sorted(VARIANTS))
def pair(request):
    cfg = VARIANTS[request.param]
    host = synth.generate(cfg)
    m = rf.Model.from_synthetic(host)
    yield cfg, m, O.OracleModel(host)
    m.close()


def test_parity_mode_bit_identical(pair):
    cfg, m, om = pair
    prompt = synth.random_prompt(cfg, 48, seed=2)
    want, want_h = om.context(128).eval(prompt, want_hidden=True)
    ctx = m.context(128, kv="f32", attn_exact=True)
    ctx.set_trace(True)
    got = ctx.eval(prompt)
    for l in range(cfg.n_layer + 1):
        h = ctx.hidden(l)
        assert np.array_equal(h.view(np.uint32), want_h[l].view(np.uint32)), (
            f"{cfg.name} layer {l}: rel L2 {rel_l2(h, want_h[l]):.3g}")
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    ctx.close()


def test_parity_mode_greedy(pair):
    cfg, m, om = pair
    prompt = synth.random_prompt(cfg, 32, seed=4)
    want = O.greedy_generate(om, prompt, 48, 128)
    got = rf.greedy_generate(m, prompt, 48, 128, kv="f32", attn_exact=True)
    assert np.array_equal(got, want), f"first divergence at {np.argmax(got != want)}"


def test_production_mode_bit_identical(pair):
    """fp16 cache and the tile attention, against the oracle with the same
    cache rounding and tile order: every layer and the logits bit for bit."""
    cfg, m, om = pair
    prompt = synth.random_prompt(cfg, 48, seed=6)
    want, want_h = om.context(128, kv_fp16=True, attn_tiles=m.attn_tiles).eval(prompt, want_hidden=True)
    ctx = m.context(128, kv="f16")
    ctx.set_trace(True)
    got = ctx.eval(prompt)
    for l in range(cfg.n_layer + 1):
        h = ctx.hidden(l)
        assert np.array_equal(h.view(np.uint32), want_h[l].view(np.uint32)), (
            f"{cfg.name} layer {l}: rel L2 {rel_l2(h, want_h[l]):.3g}")
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    ctx.close()
