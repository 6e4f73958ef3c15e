"""Tensor-parallel decode with the exchanges over peer memory
(foxcuda_tp_p2p_*, TPContext(exchange="p2p")) against the single-GPU decode,
bit for bit.

The one-GPU case runs the exchange kernels with a single rank (each slot
written and read in the rank's own arena). By default the absmax exchange and
the readiness signal run inside the terms GEMV (two launches per
row-parallel projection); one test keeps them in kernels of their own
(FOXCUDA_TP_P2P_FUSED=0), and one launches the GEMVs and the head with
programmatic stream serialisation (FOXCUDA_TP_PDL=1). The two-GPU case maps the peer's
arena through CUDA IPC. The same harness as test_tp_gpu.py applies: ranks
are child processes, and the parent fails as soon as one exits abnormally.
"""
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


def run_rank(rank, world, port, cfg, kv, exact, graphs, out_q, exchange="p2p", penalty=1.0, fused=True,
             pdl=False):
    import datetime
    import os
    # read once by the library, at the first exchange and the first launch
    os.environ["FOXCUDA_TP_P2P_FUSED"] = "1" if fused else "0"
    os.environ["FOXCUDA_TP_PDL"] = "1" if pdl else "0"
    import torch.distributed as dist
    import rustfox_b200 as rf
    from rustfox_b200.tp import TPContext
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        m = rf.Model.from_synthetic(synth.generate(cfg), device=rank, tp_rank=rank, tp_size=world)
        ctx = TPContext(m, N_CTX, kv=kv, attn_exact=exact, exchange=exchange, repeat_penalty=penalty)
        toks = ctx.generate(PROMPT, N_GEN, graphs=graphs)
        torch.cuda.synchronize()
        dist.barrier()  # no rank unmaps while another may still read its arena
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


def _tp_tokens(cfg, kv, exact, graphs, world, limit_s=240, exchange="p2p", penalty=1.0, fused=True,
               pdl=False):
    import queue
    import time
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=run_rank,
                         args=(r, world, port, cfg, kv, exact, graphs, q, exchange, penalty, fused, pdl))
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


@pytest.mark.parametrize("world", [1, 2])
def test_p2p_separate_exchange_kernels_equal_one_gpu(world):
    """FOXCUDA_TP_P2P_FUSED=0: the absmax exchange and the readiness signal in
    kernels of their own, four launches per row-parallel projection."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import rustfox_b200 as rf
    got = _tp_tokens(CFG_TQ2, "f16", False, True, world, fused=False)
    m = rf.Model.from_synthetic(synth.generate(CFG_TQ2))
    want = rf.greedy_generate(m, PROMPT, N_GEN, N_CTX, kv="f16", repeat_penalty=1.0)
    m.close()
    assert np.array_equal(got, want), f"first divergence at {np.argmax(got != want)}"


@pytest.mark.parametrize("world", [1, 2])
@pytest.mark.parametrize("graphs", [False, True], ids=["eager", "graph"])
def test_p2p_programmatic_launch_equal_one_gpu(world, graphs):
    """FOXCUDA_TP_PDL=1: the GEMVs and the head overlap their predecessors
    (the fold releases them at its start), in parity and production mode."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import rustfox_b200 as rf
    for kv, exact in (("f32", True), ("f16", False)):
        got = _tp_tokens(CFG_TQ2, kv, exact, graphs, world, pdl=True)
        m = rf.Model.from_synthetic(synth.generate(CFG_TQ2))
        want = rf.greedy_generate(m, PROMPT, N_GEN, N_CTX, kv=kv, repeat_penalty=1.0, attn_exact=exact)
        m.close()
        assert np.array_equal(got, want), f"{kv}: first divergence at {np.argmax(got != want)}"
