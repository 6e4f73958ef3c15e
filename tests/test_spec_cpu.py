"""The speculative acceptance loop (rustfox_b200/spec.py) on a stand-in
context: its tokens must equal plain greedy decoding for every seed, drafts
must sometimes be accepted, and the context must end where greedy decoding
leaves it. The device form of eval_all and rewind is tested on the GPU."""
import numpy as np
import pytest

from rustfox_b200.spec import ngram_draft, speculative_greedy


class ToyContext:
    """A seeded toy language model: the next-token logits depend on the last
    two tokens of the context, and the context can rewind."""

    def __init__(self, vocab: int, seed: int):
        rng = np.random.default_rng(seed)
        self.table = rng.normal(0, 1, (vocab, vocab, vocab)).astype(np.float32)
        self.toks = []
        self.max_pos = 0

    @property
    def pos(self):
        return len(self.toks)

    def _logits(self):
        a = self.toks[-2] if len(self.toks) > 1 else 0
        return self.table[a, self.toks[-1]].copy()

    def eval(self, tokens):
        self.toks += [int(t) for t in tokens]
        self.max_pos = max(self.max_pos, self.pos)
        return self._logits()

    def eval_all(self, tokens):
        rows = []
        for t in tokens:
            self.toks.append(int(t))
            rows.append(self._logits())
        self.max_pos = max(self.max_pos, self.pos)
        return np.stack(rows)

    def rewind(self, pos):
        assert pos <= self.pos
        del self.toks[pos:]


def plain_greedy(ctx, prompt, n_gen):
    out = [int(np.argmax(ctx.eval(prompt)))]
    while len(out) < n_gen:
        out.append(int(np.argmax(ctx.eval([out[-1]]))))
    return np.array(out, dtype=np.uint32)


@pytest.mark.parametrize("seed", range(12))
def test_speculative_equals_plain_greedy(seed):
    vocab, n_gen, k = 7, 40, 4
    prompt = np.random.default_rng(100 + seed).integers(0, vocab, 6)
    want = plain_greedy(ToyContext(vocab, seed), prompt, n_gen)
    ctx = ToyContext(vocab, seed)
    got, stats = speculative_greedy(ctx, prompt, n_gen, k=k)
    assert np.array_equal(got, want)
    # the context holds the prompt and every token but the last pick
    assert ctx.toks == [int(t) for t in prompt] + [int(t) for t in got[:-1]]
    assert ctx.max_pos <= len(prompt) + n_gen + k
    assert stats["accepted"] <= stats["drafted"]


def test_drafts_are_accepted_on_repetitive_text():
    total = 0
    for seed in range(12):
        prompt = np.random.default_rng(100 + seed).integers(0, 7, 6)
        _, stats = speculative_greedy(ToyContext(7, seed), prompt, 40, k=4)
        total += stats["accepted"]
    assert total > 0


def test_ngram_draft_takes_the_latest_match_of_the_longest_suffix():
    h = [1, 2, 3, 9, 1, 2, 3, 4, 5, 1, 2, 3]
    assert ngram_draft(h, 2) == [4, 5]          # latest "1 2 3" before the end
    assert ngram_draft([5, 6, 7], 3) == []      # nothing recurs
    assert ngram_draft([4, 4, 4], 3) == [4]     # overlap: the token after "4 4"
    assert ngram_draft(h, 0) == []
