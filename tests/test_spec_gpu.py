"""Speculative decoding on the device (rustfox_b200/spec.py over
foxcuda_eval_all and foxcuda_context_rewind) against plain greedy decoding,
token for token.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from rustfox_b200 import formats as F, synth  # noqa: E402
from rustfox_b200.spec import speculative_greedy  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

TINY = synth.CONFIGS["tiny"]
CFGS = {
    "tq2": TINY.scaled(name="tiny-spec-tq2", n_layer=3, linear_type=F.TQ2_0),
    "q4k": TINY.scaled(name="tiny-spec-q4k", n_layer=3, linear_type=F.Q4_K, attn_v_type=F.Q6_K,
                       output_type=F.Q6_K, linear_sigma=0.01),
}


@pytest.mark.parametrize("name", sorted(CFGS))
def test_speculative_equals_greedy(name):
    cfg = CFGS[name]
    m = rf.Model.from_synthetic(synth.generate(cfg))
    prompt = synth.random_prompt(cfg, 12, seed=4)
    want = rf.greedy_generate(m, prompt, 48, 96, repeat_penalty=1.0)
    ctx = rf.Context(m, 96)
    got, stats = speculative_greedy(ctx, prompt, 48, k=4)
    assert np.array_equal(got, want), (got, want, stats)
    ctx.close()
    m.close()


def test_rewind_then_eval_equals_fresh_eval():
    cfg = CFGS["tq2"]
    m = rf.Model.from_synthetic(synth.generate(cfg))
    prompt = synth.random_prompt(cfg, 10, seed=5)
    a = rf.Context(m, 64)
    a.eval(prompt)
    a.eval([1, 2, 3])
    a.rewind(len(prompt))
    got = a.eval([7]).view(np.uint32)
    b = rf.Context(m, 64)
    b.eval(prompt)
    want = b.eval([7]).view(np.uint32)
    assert np.array_equal(got, want)
    with pytest.raises(rf.FoxError):
        a.rewind(a.pos + 1)
    a.close()
    b.close()
    m.close()
