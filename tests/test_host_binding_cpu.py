"""The upstream host bound to libfoxcuda at link time (rustfox_b200/host).

Upstream's sources are compiled where they lie with fox_cuda_bind.c and
--wrap of fox_context_create / destroy / reset, fox_eval, fox_context_position
and fox_context_last_eval_seconds (include/fox/fox.h:441-450). On the CPU the
binaries must export the wrappers, resolve libfoxcuda.so in-tree, and with
FOX_CUDA=0 run upstream's own CPU path: the `fox run --temp 0` loop on ids
picks what the oracle picks (the upstream sources take the parity flags).
The build needs the upstream tree (`make -C rustfox_b200/host REF=<tree>`,
run by __graft_entry__.build()); without it these tests skip.
"""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as O
from rustfox_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD = os.path.join(ROOT, "rustfox_b200", "host", "_build")
IDS = os.path.join(BUILD, "fox_cuda_ids")
CLI = os.path.join(BUILD, "fox_cuda")
pytestmark = pytest.mark.skipif(not os.path.exists(IDS), reason="host binding not built (needs the upstream tree)")

CFG = synth.CONFIGS["tiny"].scaled(name="tiny-bind", n_layer=2)
WRAPPED = ["fox_context_create", "fox_context_destroy", "fox_context_reset", "fox_eval",
           "fox_context_position", "fox_context_last_eval_seconds"]


def run_ids(path, n_ctx, n_gen, prompt, **env):
    e = dict(os.environ, **env)
    r = subprocess.run([IDS, path, str(n_ctx), str(n_gen), *[str(int(t)) for t in prompt]],
                       capture_output=True, text=True, env=e, timeout=300)
    return r


@pytest.fixture(scope="module")
def gguf(tmp_path_factory):
    model = synth.generate(CFG)
    path = synth.write_gguf(model, str(tmp_path_factory.mktemp("bind") / "tiny.gguf"), tokenizer=True)
    return model, path


def test_binaries_wrap_the_context_api():
    for b in (IDS, CLI):
        syms = subprocess.run(["nm", b], capture_output=True, text=True, check=True).stdout
        for name in WRAPPED:
            assert f" T __wrap_{name}" in syms, (b, name)
        assert " U foxcuda_eval" in syms and " U foxcuda_context_create" in syms
        libs = subprocess.run(["ldd", b], capture_output=True, text=True).stdout
        line = next(l for l in libs.splitlines() if "libfoxcuda.so" in l)
        assert os.path.realpath(line.split("=>")[1].split("(")[0].strip()) == \
            os.path.realpath(os.path.join(ROOT, "rustfox_b200", "libfoxcuda.so"))


def test_cpu_path_picks_what_the_oracle_picks(gguf):
    model, path = gguf
    prompt = synth.random_prompt(CFG, 12, seed=5)
    r = run_ids(path, 64, 24, prompt, FOX_CUDA="0")
    assert r.returncode == 0, r.stderr
    got = np.array([int(t) for t in r.stdout.split()], dtype=np.uint32)
    want = O.greedy_generate(O.OracleModel(model), prompt, 24, 64)
    assert np.array_equal(got, want), (got.tolist(), want.tolist())
    assert "position 35" in r.stderr  # 12 prompt ids + 23 decode steps


def test_cuda_path_fails_loudly_without_a_gpu(gguf):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    _, path = gguf
    r = run_ids(path, 64, 4, synth.random_prompt(CFG, 4, seed=6))
    assert r.returncode != 0
    assert "cuda" in r.stderr.lower()
