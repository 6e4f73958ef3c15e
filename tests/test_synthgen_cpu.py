"""Synthetic weights generated on the device (foxcuda_model_upload_synthetic),
checked on the CPU through the numpy restatement in synthgen_mirror.py:
the distributions are the synthetic configs' (uniform ternary codes, fp16
block scales |N(0, sigma)|, Q8_0 of N(0, sigma), uniform K-quant bytes), the
bytes depend only on the seed, and the tensor list is synth.generate's. The
device bytes themselves are compared with the mirror on a B200
(tests/pending_synthgen_gpu.py).
"""
import ctypes

import numpy as np
import pytest

import rustfox_b200 as rf
from rustfox_b200 import api, formats as F, synth

import synthgen_mirror as M


def test_ternary_codes_are_uniform_and_scales_half_normal():
    b = M.blocks(F.TQ2_0, 64, 4096, seed=7, sigma=0.02).reshape(-1, 66)
    codes = np.stack([(b[:, :64] >> s) & 3 for s in (0, 2, 4, 6)]).reshape(-1)
    counts = np.bincount(codes, minlength=4)
    assert counts[3] == 0
    assert np.allclose(counts[:3] / codes.size, 1 / 3, atol=0.005)
    d = b[:, 64:66].copy().view(np.float16).astype(np.float64).reshape(-1)
    assert (d >= 0).all()
    assert abs(d.mean() - 0.02 * np.sqrt(2 / np.pi)) < 0.02 * 0.1


def test_tq1_0_bytes_encode_uniform_trits():
    b = M.blocks(F.TQ1_0, 64, 4096, seed=9, sigma=0.02).reshape(-1, 54)
    enc5, enc4 = {int(v): i for i, v in enumerate(F.TQ1_ENC5)}, {int(v): i for i, v in enumerate(F.TQ1_ENC4)}
    v5 = np.array([enc5[int(x)] for x in b[:200, :48].reshape(-1)])  # every qs byte is an encoding
    v4 = np.array([enc4[int(x)] for x in b[:200, 48:52].reshape(-1)])
    trits = np.concatenate([(v5 // 3**k) % 3 for k in range(5)] + [(v4 // 3**k) % 3 for k in range(4)])
    assert np.allclose(np.bincount(trits, minlength=3) / trits.size, 1 / 3, atol=0.01)
    d = b[:, 52:54].copy().view(np.float16).astype(np.float64).reshape(-1)
    assert abs(d.mean() - 0.02 * np.sqrt(2 / np.pi)) < 0.02 * 0.1


def test_q8_0_values_are_normal():
    b = M.blocks(F.Q8_0, 256, 4096, seed=3, sigma=0.02).reshape(-1, 34)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    x = (q * d).reshape(-1)
    assert abs(x.mean()) < 0.02 * 0.01 and abs(x.std() / 0.02 - 1) < 0.02
    assert np.abs(q).max(axis=1).min() >= 126  # each block's largest value maps near +-127


@pytest.mark.parametrize("tt", [F.Q4_K, F.Q6_K])
def test_k_quant_bytes_are_uniform_with_half_normal_scales(tt):
    blk, bb = F.BLOCK[tt]
    b = M.blocks(tt, 64, 4096, seed=11, sigma=0.01).reshape(-1, bb)
    body = b[:, 4:144] if tt == F.Q4_K else b[:, :208]
    assert abs(body.astype(np.float64).mean() - 127.5) < 1.0
    d = b[:, 0:2].copy() if tt == F.Q4_K else b[:, 208:210].copy()
    d = d.view(np.float16).astype(np.float64)
    assert abs(d.mean() - 0.01 * np.sqrt(2 / np.pi)) < 0.01 * 0.1


def test_bytes_depend_on_the_seed_only():
    a = M.blocks(F.TQ2_0, 8, 512, seed=5, sigma=0.02)
    assert np.array_equal(a, M.blocks(F.TQ2_0, 8, 512, seed=5, sigma=0.02))
    assert not np.array_equal(a, M.blocks(F.TQ2_0, 8, 512, seed=6, sigma=0.02))
    # a taller tensor starts with the same blocks (counters, not a stream)
    assert np.array_equal(a, M.blocks(F.TQ2_0, 16, 512, seed=5, sigma=0.02)[:a.size])


def test_tensor_list_is_generates():
    cfg = synth.CONFIGS["tiny"].scaled(n_layer=2)
    host = synth.generate(cfg)
    specs = list(synth.tensor_specs(cfg))
    assert [s[0] for s in specs] == list(host.tensors)
    for name, tt, ne, _ in specs:
        assert host.tensors[name][:2] == (tt, ne)
    seeds = {synth.device_seed(cfg.seed, i) for i in range(len(specs))}
    assert len(seeds) == len(specs)


def test_upload_synthetic_checks_its_arguments():
    L = rf.lib()
    assert L.foxcuda_model_upload_synthetic(None, 4, 0, F.TQ2_0, 256, 8, 1, 0.02) == api.ERR_ARG
    assert rf.last_error()
    h = ctypes.c_void_p()
    mi = api.ModelInfo(1, 256, 2, 1, 256, 128, 64, 1e-5, 1e4)
    if L.foxcuda_model_create_tp(ctypes.byref(mi), 0, 0, 1, ctypes.byref(h)) != api.OK:
        pytest.skip("no GPU: the model-level checks need a model")
    try:
        assert L.foxcuda_model_upload_synthetic(h, 4, 0, F.F16, 256, 8, 1, 0.02) == api.ERR_UNSUPPORTED
        assert L.foxcuda_model_upload_synthetic(h, 4, 0, F.TQ2_0, 300, 8, 1, 0.02) == api.ERR_ARG
        assert L.foxcuda_model_upload_synthetic(h, 4, 0, F.TQ2_0, 256, 8, 1, 0.0) == api.ERR_ARG
        assert L.foxcuda_model_upload_synthetic(h, 4, 5, F.TQ2_0, 256, 8, 1, 0.02) == api.ERR_ARG
    finally:
        L.foxcuda_model_destroy(h)
