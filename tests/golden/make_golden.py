"""Regenerates the golden fixtures in this directory from the upstream RustFox
library compiled from its own sources (oracle/_ref/libfoxref.so, built by
`make -C oracle ref` where the upstream tree is available).

    python tests/golden/make_golden.py

kernels.npz       per weight type: a small seeded matrix, an activation vector
                  and upstream fox_gemv's output; upstream's quantiser on one
                  vector
tiny_forward.npz  the tiny benchmark model (regenerated from its seed; a digest
                  of its bytes is stored): a 24-token prompt, upstream fox_eval's
                  logits for it and 16 greedy tokens of `fox run --temp 0`
"""
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402
from rustfox_b200 import formats as F, synth  # noqa: E402


def main():
    ref = O.RefLib()
    rng = np.random.default_rng(20261201)
    out = {}
    for tt, rows, cols in [(F.TQ1_0, 8, 2560), (F.TQ2_0, 8, 5120), (F.Q4_K, 8, 4096),
                           (F.Q6_K, 8, 4096), (F.Q8_0, 8, 2560)]:
        k = F.TYPE_NAMES[tt]
        w = F.random_blocks(rng, tt, rows, cols, 0.02)
        x = rng.normal(0, 1, cols).astype(np.float32)
        out.update({f"{k}_w": w, f"{k}_x": x, f"{k}_rows": rows, f"{k}_cols": cols,
                    f"{k}_out": ref.gemv(tt, x, w, rows, cols)})
    qx = rng.normal(0, 2, 1000).astype(np.float32)
    q, s = ref.quantize_i8(qx)
    out.update(quant_x=qx, quant_q=q, quant_scale=np.float32(s))
    np.savez_compressed(os.path.join(HERE, "kernels.npz"), **out)

    model = synth.generate(synth.CONFIGS["tiny"])
    prompt = synth.random_prompt(model.cfg, 24, seed=3)
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_gguf(model, os.path.join(d, "tiny.gguf"))
        toks, logits = ref.greedy_generate(path, prompt, 16, 64, model.cfg.n_vocab, n_threads=4)
    digest = np.frombuffer(model.tensors["blk.0.attn_q.weight"][2][:64].tobytes(), np.uint8)
    np.savez_compressed(os.path.join(HERE, "tiny_forward.npz"), model_digest=digest,
                        prompt=prompt, logits=logits, greedy=toks)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
