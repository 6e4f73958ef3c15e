"""The sharded greedy pick with repeat penalty (foxcuda_tp_set_penalty,
tp_penalty_kernel / tp_argmax_kernel / tp_pick_kernel in
rustfox_b200/csrc/ops.cuh) restated in numpy, against the oracle's sampler,
which is pinned against upstream's (tests/test_oracle.py).

Each shard penalises, at its local index, the distinct history tokens whose
rows it holds, c-fold for a token seen c times. It then takes its first
strict maximum, and the pick is the first strict maximum over the shards'
{value, global index} pairs. That must be upstream's pick over the whole
penalised vocabulary for any split, ties included.
"""
import numpy as np
import pytest

from oracle import oracle as O


def shard_penalise(logits, hist, vocab0, penalty):
    out = logits.copy()
    seen = set()
    for tok in hist:
        if tok in seen or not (vocab0 <= tok < vocab0 + out.size):
            continue
        seen.add(tok)
        c = hist.count(tok)
        v = np.float32(out[tok - vocab0])
        for _ in range(c):
            v = np.float32(v / np.float32(penalty)) if v > 0 else np.float32(v * np.float32(penalty))
        out[tok - vocab0] = v
    return out


def sharded_pick(logits, hist, bounds, penalty):
    pairs = []
    for v0, v1 in zip(bounds[:-1], bounds[1:]):
        local = shard_penalise(logits[v0:v1], hist, v0, penalty)
        i = int(np.argmax(local))          # first maximum of the shard
        pairs.append((local[i], v0 + i))
    best = pairs[0]
    for v, i in pairs[1:]:                 # first strict maximum, ties to the lower index
        if v > best[0] or (v == best[0] and i < best[1]):
            best = (v, i)
    return best[1]


@pytest.mark.parametrize("seed", range(20))
@pytest.mark.parametrize("world", [2, 3, 8])
def test_sharded_penalty_pick_equals_the_sampler(seed, world):
    rng = np.random.default_rng(seed * 10 + world)
    n_vocab, last_n, penalty = 997, 64, 1.1
    logits = rng.normal(0, 1, n_vocab).astype(np.float32)
    # history: repeats, and tokens near the maximum so the penalty decides
    top = list(np.argsort(-logits)[:6])
    hist = [int(t) for t in rng.choice(top + list(rng.integers(0, n_vocab, 20)), size=40)]
    if seed % 4 == 0:  # ties across shard borders
        logits[top[1]] = logits[top[0]]
    bounds = [0] + sorted(rng.choice(np.arange(1, n_vocab), size=world - 1, replace=False).tolist()) + [n_vocab]
    smp = O.OracleSampler(n_vocab, temperature=0.0, repeat_penalty=penalty, repeat_last_n=last_n)
    for t in hist:
        smp.accept(t)
    want = smp.pick(logits)
    got = sharded_pick(logits, hist[-last_n:], bounds, penalty)
    assert got == want
