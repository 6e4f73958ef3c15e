"""The slot protocol of the tensor-parallel exchanges over peer memory
(rustfox_b200/csrc/p2p.cuh), played out on the CPU: threads stand in for the
ranks and share arenas with the same slots, epochs and readiness flags, with
random delays between steps.

What must hold is what the device code relies on:
- every exchange reads each rank's value of its own epoch, never a later
  one. A rank overwrites a slot of a given phase only after an exchange that
  every rank reaches after reading it;
- the fold, reading every rank's terms in rank then block order, gives the
  unsharded in-order sum bit for bit.

Each rank's step follows foxcuda_tp_p2p_row and foxcuda_tp_p2p_pick: publish
the absmax into every arena, wait for all ranks' absmax in its own arena,
write its terms, signal ready into every arena, wait for all ranks' ready,
fold. The pick publishes a {value, index} pair, waits, and takes the first
strict maximum.

The device (gemv.cuh and slice.cuh PRO_XAMAX with the EPI_TERMS readiness
count) runs the first three steps inside one kernel: every CTA, a thread
here, publishes the same absmax and waits for all ranks' slots, writes the
terms of its own rows, and counts itself done; the CTA that counts last
publishes readiness. The fold starts after every CTA has finished (stream
order: the threads are joined).
"""
import random
import threading
import time

import numpy as np
import pytest

TPX_MAX = 8


def _epoch(pos, phase):
    return ((pos + 1) << 8) | phase


class Arena:
    def __init__(self, rows, stride):
        self.amax = np.zeros((2, TPX_MAX), dtype=np.uint64)
        self.pick = np.zeros((TPX_MAX, 2), dtype=np.uint64)
        self.ready = np.zeros((2, TPX_MAX), dtype=np.uint32)
        self.terms = [np.zeros((rows, stride), dtype=np.float32) for _ in range(2)]


def _wait(cond, what, limit=5.0):
    t0 = time.time()
    while not cond():
        if time.time() - t0 > limit:
            raise TimeoutError(what)
        time.sleep(0)


def _trade_amax(arenas, world, r, which, ep, value):
    """Publish this rank's absmax into every arena, then the largest of all
    ranks' slots of this epoch in the own arena."""
    word = (ep << 32) | int(np.float32(value).view(np.uint32))
    for k in range(world):
        arenas[k].amax[which, r] = np.uint64(word)
    g = np.float32(0)
    for k in range(world):
        _wait(lambda: int(arenas[r].amax[which, k]) >> 32 >= ep, "amax")
        w = int(arenas[r].amax[which, k])
        assert w >> 32 == ep, f"rank {r} saw a later absmax epoch"
        g = max(g, np.uint32(w & 0xffffffff).view(np.float32))
    return g


def _run(world, n_layer, n_tok, rows, blocks, seed, fused=False, ctas=3, count_early=False):
    rng = np.random.default_rng(seed)
    # per (token, layer, which): every rank's shard absmax and block terms
    amax = rng.random((n_tok, n_layer, 2, world)).astype(np.float32)
    terms = rng.normal(0, 1, (n_tok, n_layer, 2, world, rows, blocks)).astype(np.float32)
    picks = rng.normal(0, 1, (n_tok, world)).astype(np.float32)
    arenas = [Arena(rows, blocks) for _ in range(world)]
    out = [dict() for _ in range(world)]
    errors = []

    def fused_kernel(r, pos, layer, which, ep, rnd):
        """One launch of the fused terms GEMV on rank r: `ctas` CTAs, each
        with its own rows, a shared completion counter."""
        count = [0]
        lock = threading.Lock()
        seen = []
        cta_errors = []
        bounds = np.linspace(0, rows, ctas + 1).astype(int)

        def cta(j):
            try:
                time.sleep(rnd.random() * 1e-4)
                seen.append(_trade_amax(arenas, world, r, which, ep, amax[pos, layer, which, r]))
                lo, hi = bounds[j], bounds[j + 1]

                def write():
                    arenas[r].terms[which][lo:hi] = terms[pos, layer, which, r, lo:hi]

                if not count_early:
                    time.sleep(rnd.random() * 1e-4)
                    write()
                with lock:   # atomicAdd on the counter
                    last = count[0] == ctas - 1
                    count[0] += 1
                if last:     # the last CTA rearms the counter and publishes
                    count[0] = 0
                    for k in range(world):
                        arenas[k].ready[which, r] = np.uint32(ep)
                if count_early:  # planted: terms written after the count
                    time.sleep(5e-3)
                    write()
            except BaseException as e:  # noqa: BLE001
                cta_errors.append(e)

        ts = [threading.Thread(target=cta, args=(j,)) for j in range(ctas)]
        for t in ts:
            t.start()
        for t in ts:
            t.join(timeout=60)
        if cta_errors:
            raise cta_errors[0]
        assert len(set(float(g) for g in seen)) == 1, "the CTAs of one launch saw different absmax"
        return seen[0]

    def rank_main(r):
        rnd = random.Random(seed * 31 + r)
        try:
            for pos in range(n_tok):
                for layer in range(n_layer):
                    for which in (0, 1):
                        phase = 2 * layer + which + 1
                        ep = _epoch(pos, phase)
                        time.sleep(rnd.random() * 1e-4)
                        if fused:
                            out[r][("amax", pos, layer, which)] = fused_kernel(r, pos, layer, which, ep, rnd)
                        else:
                            # amax_x_kernel, the terms GEMV, signal_x_kernel
                            out[r][("amax", pos, layer, which)] = _trade_amax(
                                arenas, world, r, which, ep, amax[pos, layer, which, r])
                            time.sleep(rnd.random() * 1e-4)
                            arenas[r].terms[which][:] = terms[pos, layer, which, r]
                            for k in range(world):
                                arenas[k].ready[which, r] = np.uint32(ep)
                        for k in range(world):   # fold_x_kernel: wait ...
                            _wait(lambda: int(arenas[r].ready[which, k]) >= ep, "ready")
                            assert int(arenas[r].ready[which, k]) == ep, f"rank {r} saw a later ready epoch"
                        acc = np.zeros(rows, dtype=np.float32)
                        for k in range(world):   # ... then rank order, block order
                            t = arenas[k].terms[which]
                            for j in range(blocks):
                                acc = (acc + t[:, j]).astype(np.float32)
                        out[r][("fold", pos, layer, which)] = acc
                ep = _epoch(pos, 255)              # pick_x_kernel
                v = int(np.float32(picks[pos, r]).view(np.uint32))
                for k in range(world):
                    arenas[k].pick[r, 0] = np.uint64((ep << 32) | v)
                    arenas[k].pick[r, 1] = np.uint64((ep << 32) | (r * 1000 + pos))
                best = None
                for k in range(world):
                    _wait(lambda: int(arenas[r].pick[k, 1]) >> 32 >= ep, "pick")
                    a, b = int(arenas[r].pick[k, 0]), int(arenas[r].pick[k, 1])
                    assert a >> 32 == ep and b >> 32 == ep, f"rank {r} saw a later pick epoch"
                    val = np.uint32(a & 0xffffffff).view(np.float32)
                    if best is None or val > best[0]:
                        best = (val, b & 0xffffffff)
                out[r][("pick", pos)] = best
        except BaseException as e:  # noqa: BLE001 - reported to the main thread
            errors.append(e)

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    return out, amax, terms, picks


def _wrong(world, n_layer, n_tok, rows, blocks, out, amax, terms, picks):
    """The (rank, what) pairs whose result is not the unsharded one."""
    bad = []
    for pos in range(n_tok):
        for layer in range(n_layer):
            for which in (0, 1):
                want_amax = np.float32(amax[pos, layer, which].max())
                want = np.zeros(rows, dtype=np.float32)
                for k in range(world):
                    for j in range(blocks):
                        want = (want + terms[pos, layer, which, k, :, j]).astype(np.float32)
                for r in range(world):
                    if out[r][("amax", pos, layer, which)] != want_amax:
                        bad.append((r, "amax", pos, layer, which))
                    if not np.array_equal(out[r][("fold", pos, layer, which)].view(np.uint32),
                                          want.view(np.uint32)):
                        bad.append((r, "fold", pos, layer, which))
        k = int(np.argmax(picks[pos]))
        for r in range(world):
            if out[r][("pick", pos)] != (picks[pos, k], k * 1000 + pos):
                bad.append((r, "pick", pos))
    return bad


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "separate"])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_exchange_protocol_reads_every_value_once_and_folds_in_order(world, fused):
    shape = (world, 3, 4, 5, 3)  # world, layers, tokens, rows, blocks
    got = _run(*shape, seed=world, fused=fused)
    assert _wrong(*shape, *got) == []


def test_a_count_taken_before_the_terms_are_written_is_caught():
    """The model of the fused kernel with a planted ordering mistake: CTAs
    count themselves done before writing their terms, so the last count
    publishes readiness over terms still missing. The check above sees the
    folds read stale terms."""
    shape = (2, 2, 2, 6, 3)
    got = _run(*shape, seed=5, fused=True, ctas=3, count_early=True)
    assert any(b[1] == "fold" for b in _wrong(*shape, *got))


# ---- the sums exchange (gemv.cuh EPI_XSUM / PRO_NFOLD, p2p.cuh) -------------
#
# Each row-parallel producer pushes its row values, each as one {epoch, value}
# word, into its own slot of every rank's sums area (one area per projection
# kind, o or down, not one per layer); nothing else is published. The
# residual is completed by the next GEMV over it (gate|up after o, the next
# layer's q|k|v after down, the head after the last layer, the position
# advance of a prompt token), which reads every rank's words until each
# carries the exchange's epoch and adds the ranks' rows in rank order. With
# ternary shards the producer trades the absmax first; K-quant shards do not,
# so the single area per kind must be safe on the interleaving of the
# completions alone: a rank pushes o of layer l only after completing down of
# layer l - 1, which needs every rank's down words, which each rank pushes
# only after completing o of layer l - 1; across tokens the last completion
# of a token plays that part, so it is made even where nothing reads the
# residual (a prompt token).

def _run_sums(world, n_layer, n_tok, rows, seed, trade, ctas=3, drop_prompt_fold=False, skip_epoch_check=False):
    rng = np.random.default_rng(seed)
    vals = rng.normal(0, 1, (n_tok, n_layer, 2, world, rows)).astype(np.float32)
    amaxes = rng.random((n_tok, n_layer, 2, world)).astype(np.float32)
    picks = [pos % 2 == 1 for pos in range(n_tok)]  # tokens with a head
    # words[k][which][rank][row] = (epoch, value), replaced whole (one access)
    words = [[[[(0, np.float32(0))] * rows for _ in range(world)] for _ in range(2)] for _ in range(world)]
    amx = [Arena(1, 1) for _ in range(world)]
    got = [dict() for _ in range(world)]
    errors = []

    def produce(r, pos, layer, which, rnd):
        ep = _epoch(pos, 2 * layer + which + 1)
        bounds = np.linspace(0, rows, ctas + 1).astype(int)
        cta_errors = []

        def cta(j):
            try:
                time.sleep(rnd.random() * 1e-4)
                if trade:
                    _trade_amax(amx, world, r, which, ep, amaxes[pos, layer, which, r])
                for row in range(bounds[j], bounds[j + 1]):
                    for k in range(world):
                        words[k][which][r][row] = (ep, vals[pos, layer, which, r, row])
            except BaseException as e:  # noqa: BLE001
                cta_errors.append(e)

        ts = [threading.Thread(target=cta, args=(j,)) for j in range(ctas)]
        for t in ts:
            t.start()
        for t in ts:
            t.join(timeout=60)
        if cta_errors:
            raise cta_errors[0]
        return (pos, layer, which)

    def complete(r, pending):
        pos, layer, which = pending
        ep = _epoch(pos, 2 * layer + which + 1)
        acc = None
        for k in range(world):
            row_vals = np.zeros(rows, dtype=np.float32)
            for row in range(rows):
                if not skip_epoch_check:
                    _wait(lambda: words[r][which][k][row][0] >= ep, "sums word")
                e, v = words[r][which][k][row]
                assert skip_epoch_check or e == ep, f"rank {r} saw a later epoch"
                row_vals[row] = v
            acc = row_vals if acc is None else (acc + row_vals).astype(np.float32)
        got[r][pending] = acc

    def rank_main(r):
        rnd = random.Random(seed * 17 + r)
        try:
            for pos in range(n_tok):
                pending = None
                for layer in range(n_layer):
                    for which in (0, 1):
                        time.sleep(rnd.random() * 1e-4)
                        if pending is not None:  # q|k|v or gate|up completes it
                            complete(r, pending)
                        pending = produce(r, pos, layer, which, rnd)
                # the head, or a prompt token's advance, completes the last
                # one (planted: the prompt token drops it)
                if picks[pos] or not drop_prompt_fold:
                    complete(r, pending)
        except BaseException as e:  # noqa: BLE001
            errors.append(e)

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    # a rank that saw a later epoch than its own, or gave up waiting
    bad = [("error", repr(e)) for e in errors]
    for r in range(world):
        for (pos, layer, which), acc in got[r].items():
            want = vals[pos, layer, which, 0].copy()
            for k in range(1, world):
                want = (want + vals[pos, layer, which, k]).astype(np.float32)
            if not np.array_equal(acc.view(np.uint32), want.view(np.uint32)):
                bad.append((r, pos, layer, which))
            ref = got[0].get((pos, layer, which))
            if ref is None or not np.array_equal(acc.view(np.uint32), ref.view(np.uint32)):
                bad.append((r, "ranks differ", pos, layer, which))
    n_reads = sum(len(g) for g in got)
    return bad, n_reads


@pytest.mark.parametrize("trade", [True, False], ids=["ternary", "kquant"])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_sums_protocol_reads_every_rows_of_their_own_step(world, trade):
    """Every completion reads each rank's rows of its own layer and token,
    in rank order, the same on every rank, with one sums area per kind."""
    n_layer, n_tok = 3, 4
    bad, n = _run_sums(world, n_layer, n_tok, rows=7, seed=world + 10 * trade, trade=trade)
    assert bad == []
    assert n == world * n_tok * 2 * n_layer  # every exchange is completed


def test_sums_without_the_epoch_check_is_caught():
    """The model with a planted mistake: the completion takes whatever words
    are there instead of waiting for its epoch. The check above sees rows
    of another step (or none yet)."""
    # the interleavings come from OS threads: seeds until the first catch
    # (a loaded host can run a few seeds without one)
    assert any(_run_sums(3, 2, 3, rows=6, seed=30 + seed, trade=False, skip_epoch_check=True)[0]
               for seed in range(40))


def test_sums_dropping_a_prompt_tokens_completion_is_caught():
    """Planted in the model: a prompt token skips its last completion. With
    K-quant shards (no absmax trade) nothing then keeps a fast rank from
    pushing the next token's o rows over those a slower rank still reads;
    the device completes it at the position advance for that reason. Seen
    as stale rows, a later epoch, or a wait that gives up."""
    assert any(_run_sums(8, 3, 6, rows=7, seed=100 + seed, trade=False, drop_prompt_fold=True)[0]
               for seed in range(40))
