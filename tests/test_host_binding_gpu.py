"""The upstream host bound to libfoxcuda at link time, on the device.

`fox_cuda_ids` runs the `fox run --temp 0` loop on ids through upstream's
public API (src/cli.c:312-361 without the tokenizer); `fox_cuda` is
upstream's CLI itself. With the binding, fox_context_create uploads the
model through upstream's weight leases and fox_eval runs the device pass:
- production mode (fp16 K/V, tile attention) picks what the library's own
  greedy decode picks on the same GGUF;
- parity mode (FOX_CUDA_PARITY=1: fp32 K/V, upstream's attention order)
  picks what the same binary picks on upstream's CPU path (FOX_CUDA=0), and
  `fox run` prints the same text both ways.
The binaries are built here from the upstream tree; without them these
tests skip.
"""
import os
import subprocess

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from rustfox_b200 import synth  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD = os.path.join(ROOT, "rustfox_b200", "host", "_build")
IDS = os.path.join(BUILD, "fox_cuda_ids")
CLI = os.path.join(BUILD, "fox_cuda")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(IDS), reason="host binding not built")]

CFG = synth.CONFIGS["tiny"].scaled(name="tiny-bind", n_layer=2)


@pytest.fixture(scope="module")
def gguf(tmp_path_factory):
    return synth.write_gguf(synth.generate(CFG), str(tmp_path_factory.mktemp("bind") / "tiny.gguf"),
                            tokenizer=True)


def ids(path, n_ctx, n_gen, prompt, **env):
    r = subprocess.run([IDS, path, str(n_ctx), str(n_gen), *[str(int(t)) for t in prompt]],
                       capture_output=True, text=True, env=dict(os.environ, **env), timeout=300)
    assert r.returncode == 0, r.stderr
    return np.array([int(t) for t in r.stdout.split()], dtype=np.uint32)


def test_device_path_picks_what_the_library_picks(gguf):
    prompt = synth.random_prompt(CFG, 20, seed=7)
    got = ids(gguf, 128, 64, prompt)
    m = rf.Model.from_gguf(gguf)
    want = rf.greedy_generate(m, prompt, 64, 128)
    m.close()
    assert np.array_equal(got, want), f"first divergence at {int(np.argmax(got != want))}"


def test_parity_mode_picks_what_upstreams_cpu_picks(gguf):
    prompt = synth.random_prompt(CFG, 20, seed=8)
    dev = ids(gguf, 128, 64, prompt, FOX_CUDA_PARITY="1")
    cpu = ids(gguf, 128, 64, prompt, FOX_CUDA="0")
    assert np.array_equal(dev, cpu), f"first divergence at {int(np.argmax(dev != cpu))}"


def test_fox_run_prints_the_same_text(gguf):
    args = [CLI, "run", gguf, "-p", "hello", "-n", "24", "--ctx", "96", "--temp", "0"]  # (the byte vocabulary has no space piece)
    out = {}
    for name, env in (("device", {"FOX_CUDA_PARITY": "1"}), ("cpu", {"FOX_CUDA": "0"})):
        r = subprocess.run(args, capture_output=True, text=True, env=dict(os.environ, **env), timeout=300)
        assert r.returncode == 0, r.stderr
        assert "gen     24 tokens" in r.stderr
        out[name] = r.stdout
    assert out["device"] == out["cpu"]
