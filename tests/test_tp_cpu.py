"""The tensor-parallel decode algorithm on CPU: two gloo ranks, each holding its
shard of the tiny model, run the sharded step with the oracle's own kernels,
with the library's shard geometry and exchange order (rustfox_b200/tp.py,
foxcuda_tp_*):

  column-parallel q/k/v (by heads), attention, gate|up (by 256-wide FFN
  blocks) and head (by vocabulary rows); row-parallel o and down: max-
  allreduce of the shard's |x| max, int8 quantisation with that global scale,
  per-block terms d * sum, all-gather, fold in block order, residual add;
  the greedy pick over the shards' {value, index} pairs.

The result must be the unsharded oracle's, bit for bit: the first logits and
the greedy tokens. The device path runs the same steps with NCCL; its GPU test
compares it with the single-GPU device decode (test_tp_gpu.py).

The sums exchange (TPContext(exchange="sums"), FOXCUDA_TP_SUMS) is restated
too: each shard folds its own blocks per row times the global activation
scale, rank 0 adds the residual, and every rank adds the ranks' rows in rank
order (an all-gather of n_embd floats here). Its logits must stay within
1e-3 relative L2 of the unsharded decode, the ranks identical.
"""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O  # noqa: E402
from rustfox_b200 import formats as F, synth  # noqa: E402

CFG = synth.CONFIGS["tiny"].scaled(name="tiny-tp", n_layer=3)
PROMPT = synth.random_prompt(CFG, 8, seed=3)
N_GEN = 6
N_CTX = 32


def shard_geometry(cfg, rank, world):
    """The shard split of foxcuda_model_create_tp."""
    hl, kvl = cfg.n_head // world, cfg.n_head_kv // world
    nbf = cfg.n_ff // 256
    fb = [(k + 1) * nbf // world - k * nbf // world for k in range(world)]
    per = (cfg.n_vocab // world + 31) // 32 * 32
    v0 = min(cfg.n_vocab, rank * per)
    return dict(q0=rank * hl * cfg.head_dim, nq=hl * cfg.head_dim, kv0=rank * kvl * cfg.head_dim,
                nkv=kvl * cfg.head_dim, hl=hl, kvl=kvl, ob=hl * cfg.head_dim // 256,
                o0=rank * hl * cfg.head_dim // 256, fb=fb, f0=rank * nbf // world, v0=v0,
                nv=min(cfg.n_vocab, v0 + per) - v0)


def rows(t, r0, n):
    tt, ne, data = t
    rb = F.row_bytes(tt, ne[0])
    return data.view(np.uint8)[r0 * rb:(r0 + n) * rb]


def col_blocks(t, b0, nb):
    tt, ne, data = t
    rb, bb = F.row_bytes(tt, ne[0]), F.row_bytes(tt, 256)
    m = data.view(np.uint8).reshape(ne[1], rb)
    return np.ascontiguousarray(m[:, b0 * bb:(b0 + nb) * bb]).reshape(-1)


def quant_global(x, amax):
    """upstream's quantiser (src/gemv.c:20-40) with a given absmax."""
    x = x.astype(np.float32)
    inv = np.float32(127.0) / np.float32(amax) if amax > 0 else np.float32(0.0)
    v = (x * inv).astype(np.float32)
    r = np.where(v < 0, (v - np.float32(0.5)), (v + np.float32(0.5))).astype(np.float32)
    return np.clip(np.trunc(r), -127, 127).astype(np.int8)


def block_scales(tt, w, n_rows, nb):
    off = 52 if tt == F.TQ1_0 else 64
    bb = F.row_bytes(tt, 256)
    b = w.reshape(n_rows * nb, bb)
    return b[:, off:off + 2].copy().view(np.float16).astype(np.float32).reshape(n_rows, nb)


def run_rank(rank, world, port, out_q, mode="terms"):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out_q.put((rank, decode_shard(rank, world, dist, mode)))
    finally:
        dist.destroy_process_group()


def decode_shard(rank, world, dist, mode="terms"):
    L = O.lib()
    L.or_rope.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p]
    L.or_softmax.argtypes = [C.c_void_p, C.c_size_t]
    L.or_silu_mul.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
    cfg = CFG
    m = synth.generate(cfg)
    g = shard_geometry(cfg, rank, world)
    E, hd, half, tt = cfg.n_embd, cfg.head_dim, cfg.head_dim // 2, cfg.linear_type
    T = m.tensors
    lay = []
    for l in range(cfg.n_layer):
        b = f"blk.{l}."
        lay.append(dict(
            an=T[b + "attn_norm.weight"][2], fn=T[b + "ffn_norm.weight"][2],
            q=rows(T[b + "attn_q.weight"], g["q0"], g["nq"]),
            k=rows(T[b + "attn_k.weight"], g["kv0"], g["nkv"]),
            v=rows(T[b + "attn_v.weight"], g["kv0"], g["nkv"]),
            o=col_blocks(T[b + "attn_output.weight"], g["o0"], g["ob"]),
            gate=rows(T[b + "ffn_gate.weight"], g["f0"] * 256, g["fb"][rank] * 256),
            up=rows(T[b + "ffn_up.weight"], g["f0"] * 256, g["fb"][rank] * 256),
            down=col_blocks(T[b + "ffn_down.weight"], g["f0"], g["fb"][rank])))
    head = rows(T["output.weight"], g["v0"], g["nv"])
    etype, _, etab = T["token_embd.weight"]
    erb = F.row_bytes(etype, E)
    th = np.array([[p * cfg.rope_base ** (-2.0 * i / hd) for i in range(half)] for p in range(N_CTX)])
    rc, rs = np.cos(th).astype(np.float32), np.sin(th).astype(np.float32)
    kc = np.zeros((cfg.n_layer, N_CTX, g["nkv"]), np.float32)
    vc = np.zeros_like(kc)
    scale = np.float32(1.0) / np.sqrt(np.float32(hd), dtype=np.float32)
    gqa = cfg.n_head // cfg.n_head_kv
    fb_max = max(g["fb"])

    def row_parallel(xin, w, nb_local, nb_all, pad):
        amax = torch.tensor([float(np.max(np.abs(xin)))], dtype=torch.float32)
        dist.all_reduce(amax, op=dist.ReduceOp.MAX)
        amax = np.float32(amax.item())
        q8 = quant_global(xin, amax)
        isum = O.block_partials(tt, q8, w, E, nb_local * 256).reshape(E, nb_local)
        terms = np.zeros((E, pad), np.float32)
        terms[:, :nb_local] = (block_scales(tt, w, E, nb_local) * isum.astype(np.float32)).astype(np.float32)
        gath = [torch.zeros(E, pad) for _ in range(world)]
        dist.all_gather(gath, torch.from_numpy(terms))
        acc = np.zeros(E, np.float32)
        for k in range(world):
            t = gath[k].numpy()
            for j in range(nb_all[k]):
                acc = (acc + t[:, j]).astype(np.float32)
        s = (amax / np.float32(127.0)).astype(np.float32) if amax > 0 else np.float32(0.0)
        return (acc * s).astype(np.float32)

    def row_parallel_sums(x, xin, w, nb_local):
        """The sums exchange: this shard's rows (its blocks in order, times
        the global scale; rank 0 adds the residual), gathered and added in
        rank order. Returns the completed residual."""
        amax = torch.tensor([float(np.max(np.abs(xin)))], dtype=torch.float32)
        dist.all_reduce(amax, op=dist.ReduceOp.MAX)
        amax = np.float32(amax.item())
        q8 = quant_global(xin, amax)
        isum = O.block_partials(tt, q8, w, E, nb_local * 256).reshape(E, nb_local)
        terms = (block_scales(tt, w, E, nb_local) * isum.astype(np.float32)).astype(np.float32)
        acc = np.zeros(E, np.float32)
        for j in range(nb_local):
            acc = (acc + terms[:, j]).astype(np.float32)
        s = (amax / np.float32(127.0)).astype(np.float32) if amax > 0 else np.float32(0.0)
        y = (acc * s).astype(np.float32)
        if rank == 0:
            y = (x + y).astype(np.float32)
        gath = [torch.zeros(E) for _ in range(world)]
        dist.all_gather(gath, torch.from_numpy(y))
        out = gath[0].numpy().copy()
        for k in range(1, world):
            out = (out + gath[k].numpy()).astype(np.float32)
        return out

    def step(token, pos, pick):
        x = O.dequant_row(etype, etab.view(np.uint8)[token * erb:(token + 1) * erb], E)
        for l, W in enumerate(lay):
            xn = O.rmsnorm(x, W["an"], cfg.rms_eps)
            q = np.ascontiguousarray(O.gemv(tt, xn, W["q"], g["nq"], E))
            k = np.ascontiguousarray(O.gemv(tt, xn, W["k"], g["nkv"], E))
            v = O.gemv(tt, xn, W["v"], g["nkv"], E)
            cp, sp = np.ascontiguousarray(rc[pos]), np.ascontiguousarray(rs[pos])
            L.or_rope(q.ctypes.data_as(C.c_void_p), g["hl"], hd, cp.ctypes.data_as(C.c_void_p), sp.ctypes.data_as(C.c_void_p))
            L.or_rope(k.ctypes.data_as(C.c_void_p), g["kvl"], hd, cp.ctypes.data_as(C.c_void_p), sp.ctypes.data_as(C.c_void_p))
            kc[l, pos], vc[l, pos] = k, v
            att = np.zeros(g["nq"], np.float32)
            for h in range(g["hl"]):
                kvh = h // gqa
                K = kc[l, :pos + 1, kvh * hd:(kvh + 1) * hd]
                V = vc[l, :pos + 1, kvh * hd:(kvh + 1) * hd]
                s = np.zeros(pos + 1, np.float32)
                for d in range(hd):
                    s = (s + (q[h * hd + d] * K[:, d]).astype(np.float32)).astype(np.float32)
                a = np.ascontiguousarray((s * scale).astype(np.float32))
                L.or_softmax(a.ctypes.data_as(C.c_void_p), a.size)
                acc = np.zeros(hd, np.float32)
                for j in range(pos + 1):
                    acc = (acc + (a[j] * V[j]).astype(np.float32)).astype(np.float32)
                att[h * hd:(h + 1) * hd] = acc
            if mode == "sums":
                x = row_parallel_sums(x, att, W["o"], g["ob"])
            else:
                x = (x + row_parallel(att, W["o"], g["ob"], [g["ob"]] * world, g["ob"])).astype(np.float32)
            xn = O.rmsnorm(x, W["fn"], cfg.rms_eps)
            nf = g["fb"][rank] * 256
            gt = np.ascontiguousarray(O.gemv(tt, xn, W["gate"], nf, E))
            up = np.ascontiguousarray(O.gemv(tt, xn, W["up"], nf, E))
            L.or_silu_mul(gt.ctypes.data_as(C.c_void_p), up.ctypes.data_as(C.c_void_p), nf)
            if mode == "sums":
                x = row_parallel_sums(x, gt, W["down"], g["fb"][rank])
            else:
                x = (x + row_parallel(gt, W["down"], g["fb"][rank], g["fb"], fb_max)).astype(np.float32)
        if not pick:
            return None, None
        xn = O.rmsnorm(x, T["output_norm.weight"][2], cfg.rms_eps)
        logits = O.gemv(T["output.weight"][0], xn, head, g["nv"], E)
        i = int(np.argmax(logits))  # first maximum (ties to the lowest index)
        pair = torch.tensor([logits[i], float(g["v0"] + i)], dtype=torch.float64)
        pairs = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(pairs, pair)
        best = max(range(world), key=lambda r: (pairs[r][0].item(), -pairs[r][1].item()))
        return int(pairs[best][1].item()), logits

    pos, toks, first = 0, [], None
    for i, t in enumerate(PROMPT):
        nxt, lg = step(int(t), pos, i + 1 == len(PROMPT))
        pos += 1
    first = lg
    toks.append(nxt)
    for _ in range(N_GEN - 1):
        nxt, _ = step(toks[-1], pos, True)
        pos += 1
        toks.append(nxt)
    return dict(tokens=toks, logits=first, v0=g["v0"])


def _two_ranks(mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000 + (7 if mode == "sums" else 0)
    procs = [ctx.Process(target=run_rank, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    import queue
    import time
    res, t0 = {}, time.time()
    try:
        while len(res) < 2:
            try:
                r, out = q.get(timeout=2)
                res[r] = out
            except queue.Empty:
                dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
                assert not dead, f"a rank exited with {dead}"
                assert time.time() - t0 < 600, "ranks did not finish in time"
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=30)
    assert res[0]["tokens"] == res[1]["tokens"]
    return res


def test_two_shards_equal_the_unsharded_decode():
    res = _two_ranks("terms")
    om = O.OracleModel(synth.generate(CFG))
    want_logits = om.context(N_CTX).eval(PROMPT)
    want = O.greedy_generate(om, PROMPT, N_GEN, N_CTX, repeat_penalty=1.0)
    got_logits = np.concatenate([res[0]["logits"], res[1]["logits"]])
    assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32))
    assert res[0]["tokens"] == [int(t) for t in want]


def test_two_shards_sums_exchange_within_1e3():
    res = _two_ranks("sums")
    om = O.OracleModel(synth.generate(CFG))
    want_logits = om.context(N_CTX).eval(PROMPT)
    want = O.greedy_generate(om, PROMPT, N_GEN, N_CTX, repeat_penalty=1.0)
    got = np.concatenate([res[0]["logits"], res[1]["logits"]]).astype(np.float64)
    rel = np.linalg.norm(got - want_logits) / np.linalg.norm(want_logits)
    assert rel <= 1e-3, rel
    assert rel > 0.0  # the partial sums are associated differently
    assert res[0]["tokens"] == [int(t) for t in want]
