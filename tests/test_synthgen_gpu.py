"""Synthetic weights generated on the device (foxcuda_model_upload_synthetic,
Model.from_synthetic_device) against the numpy restatement of the generator
(synthgen_mirror.py) uploaded from the host: the same logits bit for bit,
the same greedy tokens, and the same device bytes (their device images are
equal).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

import rustfox_b200 as rf  # noqa: E402
from rustfox_b200 import formats as F, synth  # noqa: E402

import synthgen_mirror as M  # noqa: E402

TINY = synth.CONFIGS["tiny"]
CFGS = {
    "tq1": TINY.scaled(name="tiny-dev-tq1", n_layer=2),
    "tq2": TINY.scaled(name="tiny-dev-tq2", n_layer=2, linear_type=F.TQ2_0),
    "q4k": TINY.scaled(name="tiny-dev-q4k", n_layer=2, linear_type=F.Q4_K, attn_v_type=F.Q6_K,
                       output_type=F.Q6_K, linear_sigma=0.01),
}


def _info(cfg):
    return dict(n_layer=cfg.n_layer, n_embd=cfg.n_embd, n_head=cfg.n_head, n_head_kv=cfg.n_head_kv,
                n_ff=cfg.n_ff, head_dim=cfg.head_dim, n_vocab=cfg.n_vocab, rms_eps=cfg.rms_eps,
                rope_freq_base=cfg.rope_base)


@pytest.mark.parametrize("name", sorted(CFGS))
def test_device_generated_model_equals_the_mirror(tmp_path, name):
    cfg = CFGS[name]
    dev = rf.Model.from_synthetic_device(cfg)
    host = rf.Model(_info(cfg), M.tensors(cfg))
    prompt = synth.random_prompt(cfg, 10, seed=2)
    la = dev.context(48).eval(prompt)
    lb = host.context(48).eval(prompt)
    assert np.array_equal(np.asarray(la).view(np.uint32), np.asarray(lb).view(np.uint32))
    ta = rf.greedy_generate(dev, prompt, 12, 48, repeat_penalty=1.0)
    tb = rf.greedy_generate(host, prompt, 12, 48, repeat_penalty=1.0)
    assert np.array_equal(ta, tb)
    dev.save_image(str(tmp_path / "dev.fdi"))
    host.save_image(str(tmp_path / "host.fdi"))
    assert (tmp_path / "dev.fdi").read_bytes() == (tmp_path / "host.fdi").read_bytes()
    dev.close()
    host.close()


def test_a_device_generated_shard_equals_the_mirrors(tmp_path):
    cfg = CFGS["tq2"]
    dev = rf.Model.from_synthetic_device(cfg, tp_rank=1, tp_size=2)
    host = rf.Model(_info(cfg), M.tensors(cfg), tp_rank=1, tp_size=2)
    dev.save_image(str(tmp_path / "dev.fdi"))
    host.save_image(str(tmp_path / "host.fdi"))
    assert (tmp_path / "dev.fdi").read_bytes() == (tmp_path / "host.fdi").read_bytes()
    dev.close()
    host.close()
