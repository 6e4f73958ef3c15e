"""Tensor-parallel decode on the device (two GPUs, NCCL): each rank holds its
shard, runs the foxcuda_tp_* steps with collectives on the context's stream
(rustfox_b200/tp.py), and the greedy tokens must be the single-GPU device
decode's, bit for bit, in both modes: parity (fp32 cache, upstream-order
attention, also equal to the oracle) and production (fp16 cache, cluster
attention). Skipped with fewer than two GPUs; the algorithm itself is checked
on CPU with gloo in test_tp_cpu.py.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]

from oracle import oracle as O  # noqa: E402
from rustfox_b200 import formats as F, synth  # noqa: E402

CFG = synth.CONFIGS["tiny"].scaled(name="tiny-tp", n_layer=4)
CFG_TQ2 = CFG.scaled(name="tiny-tp-tq2", linear_type=F.TQ2_0)
PROMPT = synth.random_prompt(CFG, 24, seed=5)
N_GEN = 32
N_CTX = 96


def run_rank(rank, world, port, cfg, kv, exact, graphs, out_q):
    import datetime
    import torch.distributed as dist
    import rustfox_b200 as rf
    from rustfox_b200.tp import TPContext
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        m = rf.Model.from_synthetic(synth.generate(cfg), device=rank, tp_rank=rank, tp_size=world)
        ctx = TPContext(m, N_CTX, kv=kv, attn_exact=exact)
        toks = ctx.generate(PROMPT, N_GEN, graphs=graphs)
        torch.cuda.synchronize()
        ctx.close()
        m.close()
        out_q.put((rank, [int(t) for t in toks]))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_tokens(cfg, kv, exact, graphs=False, world=2, limit_s=240):
    """Runs the ranks as child processes; fails as soon as one of them exits
    abnormally (its peers would otherwise wait in a collective) and kills
    them all after limit_s."""
    import queue
    import time
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=run_rank, args=(r, world, port, cfg, kv, exact, graphs, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res, t0 = {}, time.time()
    try:
        while len(res) < world:
            try:
                r, toks = q.get(timeout=2)
                res[r] = toks
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
        assert res[r] == res[0]
    return np.array(res[0], dtype=np.uint32)


@pytest.mark.parametrize("cfg", [CFG, CFG_TQ2], ids=["tq1", "tq2"])
@pytest.mark.parametrize("kv,exact,graphs", [("f32", True, False), ("f16", False, False),
                                             ("f16", False, True)],
                         ids=["parity", "production", "production-graph"])
def test_two_shards_equal_one_gpu(cfg, kv, exact, graphs):
    import rustfox_b200 as rf
    got = _tp_tokens(cfg, kv, exact, graphs)
    host = synth.generate(cfg)
    m = rf.Model.from_synthetic(host)
    want = rf.greedy_generate(m, PROMPT, N_GEN, N_CTX, kv=kv, repeat_penalty=1.0, attn_exact=exact)
    m.close()
    assert np.array_equal(got, want), f"first divergence at {np.argmax(got != want)}"
    if exact:
        oracle = O.greedy_generate(O.OracleModel(host), PROMPT, N_GEN, N_CTX, repeat_penalty=1.0)
        assert np.array_equal(got, oracle)
