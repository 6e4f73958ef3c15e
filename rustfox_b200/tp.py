"""Tensor-parallel greedy decode: one process per GPU, collectives over
torch.distributed (NCCL on the GPUs) or the library's own exchanges over
peer memory.

Upstream RustFox runs one process (src/threadpool.c) and has no multi-GPU
path. The sharded step follows the library's tensor-parallel steps
(include/foxcuda.h, foxcuda_tp_*): column-parallel q/k/v, attention, gate|up and
head on each shard's rows; for the row-parallel o and down projections a
max-allreduce of one float (the absmax upstream's quantiser takes over the
whole vector, src/gemv.c:20-40), an all-gather of the per-block float terms,
and a fold in upstream's block order. Every shard therefore holds the same
residual stream as the unsharded decode, bit for bit, and the picked tokens
are the unsharded greedy tokens (first strict maximum, src/sample.c:147-153).

With exchange="sums" each row-parallel projection instead pushes its n_embd
row values (this shard's blocks folded, times the whole vector's activation
scale) to every rank over peer memory, and every rank adds the ranks' rows
in rank order: one float per row and rank crosses NVLink instead of one per
block, the ranks stay identical to each other, and the result is the
single-GPU decode's up to float rounding of the partial sums (bit for bit on
one rank). This is the allreduce of the usual Megatron split, done in a
fixed order.

All library steps and collectives go on the context's CUDA stream, in the
same order on every rank.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import api


class TPShape(C.Structure):
    _fields_ = [("tp_rank", C.c_int32), ("tp_size", C.c_int32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("n_ff", C.c_uint32), ("vocab_begin", C.c_uint32),
                ("n_vocab", C.c_uint32), ("o_blocks", C.c_uint32), ("ffn_blocks", C.c_uint32 * 8),
                ("o_terms", C.c_uint32), ("down_terms", C.c_uint32)]


def shape(model: api.Model) -> TPShape:
    s = TPShape()
    api._check(api.lib().foxcuda_tp_info(model.h, C.byref(s)))
    return s


class TPContext:
    """One shard's decode state. `group` is the torch.distributed process
    group spanning the shards (default: the world)."""

    def __init__(self, model: api.Model, n_ctx: int, kv: str = "f16", attn_exact: bool = False,
                 group=None, exchange: str = "nccl", repeat_penalty: float = 1.0,
                 repeat_last_n: int = 64, open_peers: bool = True):
        """exchange: "nccl" (torch.distributed collectives between the
        library's steps), "p2p" (the library's own exchanges over peer
        memory, foxcuda_tp_p2p_*; no host collective in a step; bit for bit
        the single-GPU decode) or "sums" (peer memory, partial row sums
        added in rank order; FOXCUDA_TP_SUMS).
        repeat_penalty > 1 penalises the last repeat_last_n tokens (prompt
        and picks) in the greedy pick, as upstream's sampler does.
        open_peers=False leaves the peer arenas to open_local (every rank's
        context in this process)."""
        import torch
        import torch.distributed as dist
        if exchange not in ("nccl", "p2p", "sums"):
            raise ValueError(f"exchange is 'nccl', 'p2p' or 'sums', not {exchange!r}")
        self.exchange = exchange
        self.peer = exchange in ("p2p", "sums")
        self.dist, self.group = dist, group
        self.model = model
        self.ctx = api.Context(model, n_ctx, kv, attn_exact)
        self.shape = shape(model)
        self.world = self.shape.tp_size
        info = model.info
        self.n_layer, self.n_embd = int(info["n_layer"]), int(info["n_embd"])
        dev = torch.device("cuda", model.device)
        self.stream = torch.cuda.ExternalStream(api.lib().foxcuda_context_stream(self.ctx.h), device=dev)
        # terms per row: o shards have o_blocks blocks, down shards up to the
        # largest FFN share; 1 term per ternary block, 8 per Q4_K, 4 per Q6_K
        self.stride_o = self.shape.o_blocks * self.shape.o_terms
        self.stride_d = max(self.shape.ffn_blocks[:self.world]) * self.shape.down_terms
        f = dict(dtype=torch.float32, device=dev)
        self.amax = torch.zeros(2, **f)
        self.terms_o = torch.zeros(self.n_embd * self.stride_o, **f)
        self.terms_d = torch.zeros(self.n_embd * self.stride_d, **f)
        self.gath_o = torch.zeros(self.world * self.n_embd * self.stride_o, **f)
        self.gath_d = torch.zeros(self.world * self.n_embd * self.stride_d, **f)
        self.best = torch.zeros(2, **f)
        self.pairs = torch.zeros(2 * self.world, **f)
        api._check(api.lib().foxcuda_tp_set_penalty(self.ctx.h, float(repeat_penalty), int(repeat_last_n)))
        if self.peer:
            if open_peers:
                self._open_peers()
            else:
                api._check(api.lib().foxcuda_tp_p2p_export(self.ctx.h, (C.c_uint8 * 64)()))
            api._check(api.lib().foxcuda_tp_p2p_mode(self.ctx.h, 1 if exchange == "sums" else 0))

    @staticmethod
    def open_local(ranks: list) -> None:
        """Map every rank's arena into every rank's context, all of them
        contexts of this process (TPContext(..., open_peers=False)), in rank
        order."""
        arr = (C.c_void_p * len(ranks))(*[r.ctx.h for r in ranks])
        for r in ranks:
            api._check(api.lib().foxcuda_tp_p2p_open_local(r.ctx.h, arr))

    def _open_peers(self):
        """Every rank's exchange arena handle to every rank, then the peers
        mapped (the one host collective, at setup)."""
        L = api.lib()
        n = 64  # FOXCUDA_IPC_HANDLE_BYTES
        h = (C.c_uint8 * n)()
        api._check(L.foxcuda_tp_p2p_export(self.ctx.h, h))
        handles = [bytes(h)]
        if self.world > 1:
            handles = [None] * self.world
            self.dist.all_gather_object(handles, bytes(h), group=self.group)
        buf = (C.c_uint8 * (n * self.world)).from_buffer_copy(b"".join(handles))
        api._check(L.foxcuda_tp_p2p_open(self.ctx.h, buf))
        if self.world > 1:
            self.dist.barrier(group=self.group)

    @staticmethod
    def _p(t, off=0):
        return C.c_void_p(t.data_ptr() + off * t.element_size())

    def _allreduce_max(self, t):
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX, group=self.group)

    def _all_gather(self, out, inp):
        if self.world > 1:
            self.dist.all_gather_into_tensor(out, inp, group=self.group)
        else:
            out.copy_(inp)

    def _row_parallel(self, layer: int, which: int):
        L = api.lib()
        if self.peer:
            api._check(L.foxcuda_tp_p2p_row(self.ctx.h, layer, which))
            return
        amax = self.amax[which:which + 1]
        terms, gath, stride = ((self.terms_o, self.gath_o, self.stride_o) if which == 0
                               else (self.terms_d, self.gath_d, self.stride_d))
        api._check(L.foxcuda_tp_amax(self.ctx.h, which, self._p(amax)))
        self._allreduce_max(amax)
        api._check(L.foxcuda_tp_terms(self.ctx.h, layer, which, self._p(amax), self._p(terms), stride))
        self._all_gather(gath, terms)
        api._check(L.foxcuda_tp_fold(self.ctx.h, layer, which, self._p(gath), stride, self._p(amax)))

    def step(self, token: int | None, pick: bool):
        """One token through the shards: token from the host, or (None) the
        last pick on the device. With pick the next token is chosen."""
        import torch
        L = api.lib()
        with torch.cuda.stream(self.stream):
            api._check(L.foxcuda_tp_embed(self.ctx.h, -1 if token is None else int(token)))
            for l in range(self.n_layer):
                api._check(L.foxcuda_tp_attention(self.ctx.h, l))
                self._row_parallel(l, 0)
                api._check(L.foxcuda_tp_ffn(self.ctx.h, l))
                self._row_parallel(l, 1)
            if pick and self.peer:
                api._check(L.foxcuda_tp_p2p_pick(self.ctx.h))
            elif pick:
                api._check(L.foxcuda_tp_head(self.ctx.h, self._p(self.best)))
                self._all_gather(self.pairs, self.best)
                api._check(L.foxcuda_tp_pick(self.ctx.h, self._p(self.pairs)))
            else:
                api._check(L.foxcuda_tp_advance(self.ctx.h))

    def capture(self):
        """Record one decode step fed by the last pick (library kernels and the
        NCCL collectives) as a CUDA graph. Its inputs are all on the device
        (token, position), so each replay is the next step. Call after at
        least one eager step (attributes set, communicators created)."""
        import torch
        self.graph = torch.cuda.CUDAGraph()
        pos = self.ctx.pos
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.step(None, pick=True)
        # capture does not run the step: the host counter goes back
        self.ctx_pos_fix(pos)

    def ctx_pos_fix(self, pos=None):
        api._check(api.lib().foxcuda_context_sync_position(self.ctx.h))

    def replay(self, n: int):
        """n replays of the captured step, on the context's stream (a graph
        replays on the current stream)."""
        import torch
        with torch.cuda.stream(self.stream):
            for _ in range(n):
                self.graph.replay()
        self.ctx_pos_fix()

    def decode(self, token: int) -> int:
        """One step through the C ABI with host buffers, as a serving loop
        makes it: the token copied in from pinned host memory
        (foxcuda_tp_feed), the captured step replayed, the pick read back
        (foxcuda_tp_tokens, which synchronises: 4 bytes of token and 4 of
        error word) and the position re-read (4 bytes). Call after
        capture()."""
        import torch
        L = api.lib()
        p = self.ctx.pos
        api._check(L.foxcuda_tp_feed(self.ctx.h, int(token)))
        with torch.cuda.stream(self.stream):
            self.graph.replay()
        out = np.zeros(1, dtype=np.uint32)
        api._check(L.foxcuda_tp_tokens(self.ctx.h, p, 1, out.ctypes.data_as(C.c_void_p)))
        self.ctx_pos_fix()
        return int(out[0])

    def generate(self, prompt, n_gen: int, graphs: bool = False) -> np.ndarray:
        """Greedy decode with the context's repeat penalty (none by default):
        the prompt, then n_gen picks; with graphs the steps after the first
        two replay a captured step."""
        prompt = [int(t) for t in prompt]
        start = self.ctx.pos
        for i, t in enumerate(prompt):
            self.step(t, pick=(i + 1 == len(prompt)))
        rest = n_gen - 1
        if graphs and rest > 1:
            self.step(None, pick=True)
            rest -= 1
            if getattr(self, "graph", None) is None:
                self.capture()
            self.replay(rest)
            rest = 0
        for _ in range(rest):
            self.step(None, pick=True)
        out = np.zeros(n_gen, dtype=np.uint32)
        first = start + len(prompt) - 1
        api._check(api.lib().foxcuda_tp_tokens(self.ctx.h, first, n_gen,
                                               out.ctypes.data_as(C.c_void_p)))
        return out

    def profile_step(self) -> dict:
        """One eager step fed by the last pick with a CUDA event after every
        library call: microseconds per phase, summed over the layers
        (q|k|v + attention, o with its exchange, gate|up, down with its
        exchange, head + pick). With the sums exchange a projection's wait
        for the peers' rows lands in the phase of the GEMV that completes
        them (gate|up after o, q|k|v after down). The events end the overlap
        between phases, so the sum is above a captured step's time."""
        import torch
        L = api.lib()
        marks = []

        def mark(name):
            e = torch.cuda.Event(enable_timing=True)
            e.record(self.stream)
            marks.append((name, e))

        with torch.cuda.stream(self.stream):
            mark("start")
            api._check(L.foxcuda_tp_embed(self.ctx.h, -1))
            mark("embed")
            for l in range(self.n_layer):
                api._check(L.foxcuda_tp_attention(self.ctx.h, l))
                mark("qkv+attention")
                self._row_parallel(l, 0)
                mark("o")
                api._check(L.foxcuda_tp_ffn(self.ctx.h, l))
                mark("gate_up")
                self._row_parallel(l, 1)
                mark("down")
            if self.peer:
                api._check(L.foxcuda_tp_p2p_pick(self.ctx.h))
            else:
                api._check(L.foxcuda_tp_head(self.ctx.h, self._p(self.best)))
                self._all_gather(self.pairs, self.best)
                api._check(L.foxcuda_tp_pick(self.ctx.h, self._p(self.pairs)))
            mark("head+pick")
        self.stream.synchronize()
        out = {}
        for (_, a), (name, b) in zip(marks, marks[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b) * 1e3
        return out

    def logits(self) -> np.ndarray:
        """This shard's logits of the last picked step: vocabulary rows
        [vocab_begin, vocab_begin + n_vocab) of the whole head."""
        out = np.zeros(self.shape.n_vocab, dtype=np.float32)
        api._check(api.lib().foxcuda_context_logits(self.ctx.h, out.ctypes.data_as(C.c_void_p),
                                                    out.size))
        return out

    def close(self):
        """Releases the captured step first: a graph that holds NCCL
        collectives must be gone before the process group is destroyed."""
        g = getattr(self, "graph", None)
        if g is not None:
            import torch
            torch.cuda.synchronize()
            g.reset()
            self.graph = None
        self.ctx.close()
