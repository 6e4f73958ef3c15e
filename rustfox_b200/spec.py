"""Greedy speculative decoding: drafts checked in one verification pass.

Upstream plans speculative decoding (README.md:86-89) but has neither the
all-row logits it needs (forward_batch keeps the last row,
src/forward.c:405-408) nor an acceptance loop. Here the drafts come from the
token history itself (prompt lookup: what followed the latest earlier
occurrence of the current suffix). A draft of k tokens is checked with one
foxcuda_eval_all of k + 1 tokens. The longest prefix the greedy picks agree
with is kept, plus the pick after it, and the context is rewound past the
rest. Every kept token is the greedy pick (first strict maximum,
src/sample.c:147-153) of the logits that token-by-token decoding would
produce, so the output is plain greedy decoding's. Repeat penalty is not
applied, so this is `--temp 0` without it.

The loop needs only eval(tokens) -> last logits, eval_all(tokens) -> logits
per token, rewind(pos) and pos from its context, so it runs on a
rustfox_b200.api.Context or on any object with that interface.
"""
from __future__ import annotations

import numpy as np


def ngram_draft(history, k: int, n_max: int = 3, n_min: int = 1) -> list:
    """Up to k tokens that followed the latest earlier occurrence of the
    history's longest suffix of n_max .. n_min tokens; [] when none recurs."""
    h = list(history)
    if k <= 0:
        return []
    for n in range(n_max, n_min - 1, -1):
        if len(h) <= n:
            continue
        tail = h[-n:]
        for start in range(len(h) - n - 1, -1, -1):
            if h[start:start + n] == tail:
                follow = h[start + n:start + n + k]
                if follow:
                    return follow
    return []


def speculative_greedy(ctx, prompt, n_gen: int, k: int = 4, n_max: int = 3):
    """n_gen greedy tokens after prompt, verifying history drafts of up to k
    tokens per pass. The context needs room for len(prompt) + n_gen + k
    positions. Returns (tokens, stats)."""
    prompt = [int(t) for t in prompt]
    tok = int(np.argmax(ctx.eval(prompt)))
    out = [tok]
    stats = {"passes": 0, "steps": 0, "drafted": 0, "accepted": 0}
    while len(out) < n_gen:
        draft = ngram_draft(prompt + out, min(k, n_gen - len(out) - 1), n_max)
        if not draft:
            tok = int(np.argmax(ctx.eval([tok])))
            out.append(tok)
            stats["steps"] += 1
            continue
        start = ctx.pos
        rows = ctx.eval_all([tok] + draft)   # rows[i]: logits after the i-th of these tokens
        picks = [int(np.argmax(r)) for r in rows]
        m = 0
        while m < len(draft) and picks[m] == draft[m]:
            m += 1
        out.extend(draft[:m])
        out.append(picks[m])
        ctx.rewind(start + m + 1)           # keep tok and the accepted draft tokens
        tok = picks[m]
        stats["passes"] += 1
        stats["drafted"] += len(draft)
        stats["accepted"] += m
    return np.array(out[:n_gen], dtype=np.uint32), stats
