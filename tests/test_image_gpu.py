"""Device images on a B200: a model saved with foxcuda_model_save_image and
opened with foxcuda_model_open_image decodes exactly as the model it came
from, holds the same device bytes, and saves back to the same file.

The cases cover TQ1_0 layers (held as TQ2_0 in HBM, so the image carries the
transcoded bytes), TQ2_0, the K-quant model of config 3 (Q4_K with a Q6_K v
and head, the unit layout) and a tensor-parallel shard.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

import rustfox_b200 as rf  # noqa: E402
from rustfox_b200 import formats as F, synth  # noqa: E402

TINY = synth.CONFIGS["tiny"]
CFGS = {
    "tq1": TINY.scaled(name="tiny-image", n_layer=3),
    "tq2": TINY.scaled(name="tiny-image-tq2", n_layer=3, linear_type=F.TQ2_0),
    "q4k": TINY.scaled(name="tiny-image-q4k", n_layer=3, linear_type=F.Q4_K, attn_v_type=F.Q6_K,
                       output_type=F.Q6_K, linear_sigma=0.01),
}


@pytest.mark.parametrize("name", sorted(CFGS))
def test_an_opened_image_decodes_as_the_saved_model(tmp_path, name):
    cfg = CFGS[name]
    a = rf.Model.from_synthetic(synth.generate(cfg))
    path = tmp_path / "m.fdi"
    a.save_image(str(path))
    b = rf.Model.open_image(str(path))
    assert b.device_bytes == a.device_bytes
    for k, v in b.info.items():  # the header keeps the floats as float32
        assert np.float32(v) == np.float32(a.info[k]), k
    prompt = synth.random_prompt(cfg, 12, seed=3)
    for kv, exact in (("f32", True), ("f16", False)):
        want = rf.greedy_generate(a, prompt, 24, 64, kv=kv, repeat_penalty=1.0, attn_exact=exact)
        got = rf.greedy_generate(b, prompt, 24, 64, kv=kv, repeat_penalty=1.0, attn_exact=exact)
        assert np.array_equal(got, want), f"{kv}: first divergence at {np.argmax(got != want)}"
    ca, cb = a.context(64), b.context(64)
    la, lb = ca.eval(prompt), cb.eval(prompt)
    assert np.array_equal(np.asarray(la).view(np.uint32), np.asarray(lb).view(np.uint32))
    ca.close()
    cb.close()
    # the opened model saves back to the same bytes
    again = tmp_path / "again.fdi"
    b.save_image(str(again))
    assert path.read_bytes() == again.read_bytes()
    a.close()
    b.close()


def test_a_shard_image_keeps_its_shard(tmp_path):
    cfg = CFGS["tq2"]
    a = rf.Model.from_synthetic(synth.generate(cfg), tp_rank=1, tp_size=2)
    path = tmp_path / "s.fdi"
    a.save_image(str(path))
    b = rf.Model.open_image(str(path))
    assert (b.tp_rank, b.tp_size) == (1, 2)
    assert b.device_bytes == a.device_bytes
    again = tmp_path / "again.fdi"
    b.save_image(str(again))
    assert path.read_bytes() == again.read_bytes()
    a.close()
    b.close()
