"""Tensor-parallel decode with the exchanges over peer memory
(foxcuda_tp_p2p_*) against the single-GPU decode.

  terms (TPContext(exchange="p2p"))  bit for bit the single-GPU decode
  sums  (TPContext(exchange="sums")) bit for bit on one rank; on two ranks
        every layer's residual and the logits within 1e-3 relative L2 of
        the single-GPU decode, the ranks identical to each other

The one-GPU case runs the exchange kernels with a single rank (each slot
written and read in the rank's own arena). The GEMVs, the attention and the
head overlap their predecessors (programmatic stream serialisation), as in
the single-GPU step. The absmax exchange and the readiness signal run inside
the terms GEMV (two launches per row-parallel projection). The two-GPU case
maps the peer's arena through CUDA IPC. The same harness as
test_tp_gpu.py applies: ranks are child processes, and the parent fails as
soon as one exits abnormally.

A rank whose peer never publishes (failure detection): two shards' contexts
in one process on one GPU, only rank 0 steps; its bounded waits give up, the
host reads FOXCUDA_ERR_INTERNAL, and the context stays usable.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

from rustfox_b200 import formats as F, synth  # noqa: E402

CFG = synth.CONFIGS["tiny"].scaled(name="tiny-tp", n_layer=4)
CFG_TQ2 = CFG.scaled(name="tiny-tp-tq2", linear_type=F.TQ2_0)
PROMPT = synth.random_prompt(CFG, 24, seed=5)
N_GEN = 32
N_CTX = 96


def run_rank(rank, world, port, cfg, kv, exact, graphs, out_q, exchange="p2p", penalty=1.0, trace=False):
    import datetime
    import torch.distributed as dist
    import rustfox_b200 as rf
    from rustfox_b200.tp import TPContext
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        m = rf.Model.from_synthetic(synth.generate(cfg), device=rank, tp_rank=rank, tp_size=world)
        ctx = TPContext(m, N_CTX, kv=kv, attn_exact=exact, exchange=exchange, repeat_penalty=penalty)
        extra = None
        if trace:
            # the prompt with every layer's residual kept, then this shard's logits
            ctx.ctx.set_trace(True)
            for i, t in enumerate(PROMPT):
                ctx.step(int(t), pick=(i + 1 == len(PROMPT)))
            torch.cuda.synchronize()
            extra = {"hidden": [ctx.ctx.hidden(l) for l in range(cfg.n_layer + 1)],
                     "logits": ctx.logits(), "vocab_begin": int(ctx.shape.vocab_begin)}
            ctx.ctx.set_trace(False)
            ctx.ctx.reset()
            if ctx.peer:
                dist.barrier()  # every rank has reset before any rank's next exchange
                api_clear(ctx)
                dist.barrier()
        toks = ctx.generate(PROMPT, N_GEN, graphs=graphs)
        torch.cuda.synchronize()
        dist.barrier()  # no rank unmaps while another may still read its arena
        ctx.close()
        m.close()
        out_q.put((rank, [int(t) for t in toks], extra))
    finally:
        dist.destroy_process_group()


def api_clear(ctx):
    from rustfox_b200 import api
    api._check(api.lib().foxcuda_tp_p2p_clear(ctx.ctx.h))


def _free_port() -> int:
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_run(cfg, kv, exact, graphs, world, limit_s=240, exchange="p2p", penalty=1.0, trace=False):
    import queue
    import time
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=run_rank,
                         args=(r, world, port, cfg, kv, exact, graphs, q, exchange, penalty, trace))
             for r in range(world)]
    for p in procs:
        p.start()
    res, t0 = {}, time.time()
    try:
        while len(res) < world:
            try:
                r, toks, extra = q.get(timeout=2)
                res[r] = (toks, extra)
            except queue.Empty:
                dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
                assert not dead, f"a rank exited with {dead}"
                assert time.time() - t0 < limit_s, "ranks did not finish in time"
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=30)
    for r in range(1, world):
        assert res[r][0] == res[0][0]
    return np.array(res[0][0], dtype=np.uint32), [res[r][1] for r in range(world)]


def _tp_tokens(*a, **kw):
    return _tp_run(*a, **kw)[0]


@pytest.mark.parametrize("world", [1, 2])
@pytest.mark.parametrize("cfg", [CFG, CFG_TQ2], ids=["tq1", "tq2"])
@pytest.mark.parametrize("kv,exact,graphs", [("f32", True, False), ("f16", False, False),
                                             ("f16", False, True)],
                         ids=["parity", "production", "production-graph"])
def test_p2p_shards_equal_one_gpu(world, cfg, kv, exact, graphs):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import rustfox_b200 as rf
    got = _tp_tokens(cfg, kv, exact, graphs, world)
    m = rf.Model.from_synthetic(synth.generate(cfg))
    want = rf.greedy_generate(m, PROMPT, N_GEN, N_CTX, kv=kv, repeat_penalty=1.0, attn_exact=exact)
    m.close()
    assert np.array_equal(got, want), f"first divergence at {np.argmax(got != want)}"


@pytest.mark.parametrize("world", [1, 2])
@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
@pytest.mark.parametrize("graphs", [False, True], ids=["eager", "graph"])
def test_repeat_penalty_shards_equal_one_gpu(world, exchange, graphs):
    """foxcuda_tp_set_penalty: the sharded pick with upstream's repeat penalty
    (1.1 over the last 64 tokens, prompt included) equals the single-GPU
    sampler's."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import rustfox_b200 as rf
    got = _tp_tokens(CFG_TQ2, "f16", False, graphs, world, exchange=exchange, penalty=1.1)
    m = rf.Model.from_synthetic(synth.generate(CFG_TQ2))
    want = rf.greedy_generate(m, PROMPT, N_GEN, N_CTX, kv="f16", repeat_penalty=1.1)
    m.close()
    assert np.array_equal(got, want), f"first divergence at {np.argmax(got != want)}"


@pytest.mark.parametrize("cfg", [CFG, CFG_TQ2], ids=["tq1", "tq2"])
@pytest.mark.parametrize("kv,exact,graphs", [("f32", True, False), ("f16", False, False),
                                             ("f16", False, True)],
                         ids=["parity", "production", "production-graph"])
def test_sums_one_rank_equals_one_gpu(cfg, kv, exact, graphs):
    """The sums exchange on one rank: rank 0's row values carry the
    residual, so the completed residual is the single-GPU one bit for bit."""
    import rustfox_b200 as rf
    got = _tp_tokens(cfg, kv, exact, graphs, 1, exchange="sums")
    m = rf.Model.from_synthetic(synth.generate(cfg))
    want = rf.greedy_generate(m, PROMPT, N_GEN, N_CTX, kv=kv, repeat_penalty=1.0, attn_exact=exact)
    m.close()
    assert np.array_equal(got, want), f"first divergence at {np.argmax(got != want)}"


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("graphs", [False, True], ids=["eager", "graph"])
def test_sums_two_ranks_within_1e3_of_one_gpu(graphs):
    """Two ranks, partial row sums added in rank order: every layer's
    residual and the gathered logits within 1e-3 relative L2 of the
    single-GPU decode (the int8 activations are the same; only the float
    sums are associated differently), the ranks' tokens identical, and the
    greedy tokens the single-GPU ones for at least the first 16."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import rustfox_b200 as rf
    got, extras = _tp_run(CFG_TQ2, "f16", False, graphs, 2, exchange="sums", trace=True)
    m = rf.Model.from_synthetic(synth.generate(CFG_TQ2))
    ctx = m.context(N_CTX, kv="f16")
    ctx.set_trace(True)
    want_logits = ctx.eval(PROMPT)
    want_h = [ctx.hidden(l) for l in range(CFG_TQ2.n_layer + 1)]
    ctx.close()
    want = rf.greedy_generate(m, PROMPT, N_GEN, N_CTX, kv="f16", repeat_penalty=1.0)
    m.close()
    for r, ex in enumerate(extras):
        for l, h in enumerate(ex["hidden"]):
            assert _rel(h, want_h[l]) <= 1e-3, f"rank {r} layer {l}: {_rel(h, want_h[l]):.3g}"
        assert np.array_equal(ex["hidden"][-1].view(np.uint32), extras[0]["hidden"][-1].view(np.uint32))
    logits = np.concatenate([ex["logits"] for ex in sorted(extras, key=lambda e: e["vocab_begin"])])
    assert logits.size == want_logits.size
    assert _rel(logits, want_logits) <= 1e-3, _rel(logits, want_logits)
    n = len(got) if np.array_equal(got, want) else int(np.argmax(got != want))
    assert n >= 16, f"first divergence at {n}"


@pytest.mark.parametrize("exchange", ["p2p", "sums"])
def test_peer_that_never_publishes_is_reported(exchange):
    """Failure detection without a GPU fault: rank 1 of a two-shard model
    never steps, so no readiness or absmax of its ever arrives. Rank 0's
    bounded waits give up (the first after about a second, the rest at once
    once the context's error word is set), the host reads
    FOXCUDA_ERR_INTERNAL, and after foxcuda_tp_p2p_clear the context still
    answers. Both shards live in this process on one GPU; only rank 0
    launches anything, so no two kernels wait on each other."""
    import time
    import rustfox_b200 as rf
    from rustfox_b200 import api
    from rustfox_b200.tp import TPContext
    host = synth.generate(CFG_TQ2)
    ms = [rf.Model.from_synthetic(host, device=0, tp_rank=r, tp_size=2) for r in range(2)]
    cs = [TPContext(m, N_CTX, kv="f16", exchange=exchange, open_peers=False) for m in ms]
    TPContext.open_local(cs)
    t0 = time.time()
    cs[0].step(int(PROMPT[0]), pick=True)
    with pytest.raises(api.FoxError) as e:
        out = np.zeros(1, np.uint32)
        api._check(api.lib().foxcuda_tp_tokens(cs[0].ctx.h, 0, 1, out.ctypes.data_as(C.c_void_p)))
    took = time.time() - t0
    assert e.value.status == api.ERR_INTERNAL
    assert "did not arrive" in e.value.message
    assert took < 60, f"the failed step took {took:.1f} s"
    api._check(api.lib().foxcuda_tp_p2p_clear(cs[0].ctx.h))
    cs[0].ctx.reset()
    assert cs[0].ctx.pos == 0
    for c in cs:
        c.close()
    for m in ms:
        m.close()
