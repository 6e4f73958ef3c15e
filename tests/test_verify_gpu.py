"""The verification pass (foxcuda_eval_all): the logits of every token of a
draft, against the token-by-token decode, bit for bit.

Upstream plans speculative decoding (README.md:86-89) but its forward_batch
keeps only the last row (src/forward.c:405-408). Row t of eval_all must be
the logits fox_eval gives after token t. Drafts of two or more tokens take
the chunk path: the ternary pass for the TQ models, the K-quant pass
(Q4_K with a Q6_K v and head, as in config 3) for the third; a one-token
draft steps. In the production cases the chunk's attention is one
cluster-kernel launch per layer (grid z = token); the parity cases keep the
serial upstream-order kernel, one launch per token.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from rustfox_b200 import formats as F, synth  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

TINY = synth.CONFIGS["tiny"]
CFGS = {
    "tq1": TINY.scaled(name="tiny-verify", n_layer=3),
    "tq2": TINY.scaled(name="tiny-verify-tq2", n_layer=3, linear_type=F.TQ2_0),
    "q4k": TINY.scaled(name="tiny-verify-q4k", n_layer=3, linear_type=F.Q4_K, attn_v_type=F.Q6_K,
                       output_type=F.Q6_K, linear_sigma=0.01),
}
MODELS = {}


def _model(name):
    if name not in MODELS:
        MODELS[name] = rf.Model.from_synthetic(synth.generate(CFGS[name]))
    return MODELS[name]


@pytest.mark.parametrize("name", sorted(CFGS))
@pytest.mark.parametrize("kv,exact", [("f16", False), ("f32", True)], ids=["production", "parity"])
@pytest.mark.parametrize("n_draft", [1, 8, 70])
def test_eval_all_rows_equal_steps(name, kv, exact, n_draft):
    cfg = CFGS[name]
    model = _model(name)
    prompt = synth.random_prompt(cfg, 20, seed=1)
    draft = synth.random_prompt(cfg, n_draft, seed=2)
    a = rf.Context(model, 128, kv=kv, attn_exact=exact)
    a.eval(prompt)
    rows = a.eval_all(draft).view(np.uint32)
    b = rf.Context(model, 128, kv=kv, attn_exact=exact)
    b.eval(prompt)
    want = np.stack([b.eval([t]) for t in draft]).view(np.uint32)
    assert a.pos == b.pos == 20 + n_draft
    bad = np.argwhere(rows != want)
    assert bad.size == 0, f"{len(bad)} logits differ, first at (row, index) {tuple(bad[0])}"
    a.close()
    b.close()
