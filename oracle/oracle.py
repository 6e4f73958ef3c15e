"""ctypes access to the CPU checkers. TEST INFRASTRUCTURE ONLY.

Two checkers live under oracle/:
  liboracle.so        this repository's C restatement (foxoracle.c)
  _ref/libfoxref*.so  the upstream RustFox sources compiled from where they lie
                      (oracle/Makefile); present only where they were built

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this module, and only as the checker or the timed CPU baseline.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libfoxref.so")
REF_FAST_SO = os.path.join(HERE, "_ref", "libfoxref_fast.so")

F32, F16, Q8_0, Q4_K, Q6_K, TQ1_0, TQ2_0 = 0, 1, 8, 12, 14, 34, 35

_vp, _sz, _fp, _u32 = C.c_void_p, C.c_size_t, C.c_float, C.c_uint32


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class OrModelInfo(C.Structure):
    _fields_ = [("n_layer", _u32), ("n_embd", _u32), ("n_head", _u32),
                ("n_head_kv", _u32), ("n_ff", _u32), ("head_dim", _u32),
                ("n_vocab", _u32), ("rms_eps", _fp), ("rope_freq_base", _fp)]


class OrTensor(C.Structure):
    _fields_ = [("type", C.c_int), ("ne0", C.c_uint64), ("ne1", C.c_uint64),
                ("data", _vp)]


class OrLayer(C.Structure):
    _fields_ = [(n, OrTensor) for n in ("attn_norm", "attn_q", "attn_k", "attn_v",
                                        "attn_out", "ffn_norm", "ffn_gate", "ffn_up",
                                        "ffn_down")]


class OrModel(C.Structure):
    _fields_ = [("info", OrModelInfo), ("token_embd", OrTensor),
                ("output_norm", OrTensor), ("output", OrTensor),
                ("layers", C.POINTER(OrLayer))]


class SamplerConfig(C.Structure):
    """Same layout as upstream fox_sampler_config (include/fox/fox.h:455-462)."""
    _fields_ = [("temperature", _fp), ("top_k", C.c_int), ("top_p", _fp),
                ("repeat_penalty", _fp), ("repeat_last_n", _u32), ("seed", C.c_uint64)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"{ORACLE_SO} is missing: run `make -C oracle oracle`")
        L = C.CDLL(ORACLE_SO)
        L.or_set_exp_mode.argtypes = [C.c_int]
        L.or_expf_mismatches.restype = C.c_size_t
        L.or_expf_mismatches.argtypes = [C.c_uint32, C.c_size_t, C.c_void_p, C.POINTER(C.c_size_t)]
        L.or_f16_to_f32.restype = _fp
        L.or_f16_to_f32.argtypes = [C.c_uint16]
        L.or_f32_to_f16_rne.restype = C.c_uint16
        L.or_f32_to_f16_rne.argtypes = [_fp]
        L.or_quantize_i8.argtypes = [_vp, _sz, _vp, _vp]
        L.or_quantize_k.argtypes = [_vp, _sz, _vp, _vp]
        L.or_tq1_block_sum.restype = C.c_int32
        L.or_tq1_block_sum.argtypes = [_vp, _vp]
        L.or_tq2_block_sum.restype = C.c_int32
        L.or_tq2_block_sum.argtypes = [_vp, _vp]
        L.or_block_partials.argtypes = [C.c_int, _vp, _vp, _sz, _sz, _vp]
        L.or_gemv_tq_i8.argtypes = [C.c_int, _vp, _fp, _vp, _sz, _sz, _vp]
        L.or_gemv.argtypes = [C.c_int, _vp, _vp, _sz, _sz, _vp]
        L.or_dequant_row.argtypes = [C.c_int, _vp, _sz, _vp]
        L.or_rmsnorm.argtypes = [_vp, _vp, _vp, _sz, _fp]
        L.or_ctx_create.restype = _vp
        L.or_ctx_create.argtypes = [C.POINTER(OrModel), _u32, C.c_int]
        L.or_ctx_destroy.argtypes = [_vp]
        L.or_ctx_reset.argtypes = [_vp]
        L.or_ctx_set_attn_tiles.argtypes = [_vp, C.c_int]
        L.or_tile_attention.argtypes = [_vp, _vp, _vp, _sz, _sz, _sz, C.c_int, _fp, _vp]
        L.or_ctx_pos.restype = _u32
        L.or_ctx_pos.argtypes = [_vp]
        L.or_eval.argtypes = [_vp, _vp, _sz, _vp, _vp]
        L.or_last_error.restype = C.c_char_p
        L.or_sampler_create.restype = _vp
        L.or_sampler_create.argtypes = [C.POINTER(SamplerConfig), _sz]
        L.or_sampler_destroy.argtypes = [_vp]
        L.or_sampler_accept.argtypes = [_vp, _u32]
        L.or_sampler_pick.argtypes = [_vp, _vp, _vp]
        _lib = L
    return _lib


def _check(st: int, what: str):
    if st != 0:
        raise RuntimeError(f"oracle {what}: status {st}: {lib().or_last_error().decode()}")


def lib_expf(x: float) -> float:
    """libm's expf, as upstream calls it."""
    if not hasattr(lib_expf, "f"):
        m = C.CDLL("libm.so.6")
        m.expf.restype, m.expf.argtypes = C.c_float, [C.c_float]
        lib_expf.f = m.expf
    return lib_expf.f(x)


def expf_mismatches(first_bits: int, got: np.ndarray):
    """(count, first index) of got[i] that differ bit for bit from libm's expf
    of the float with bit pattern first_bits + i (test support)."""
    got = np.ascontiguousarray(got, dtype=np.float32)
    first = C.c_size_t(0)
    n = lib().or_expf_mismatches(int(first_bits), got.size, got.ctypes.data_as(C.c_void_p), C.byref(first))
    return int(n), int(first.value)


class exp_mode:
    """Context manager: run the oracle with libm expf (upstream's and the
    device's, False) or the correctly rounded exponential (True), a
    diagnostic of what glibc's rounding alone changes."""

    def __init__(self, correctly_rounded: bool):
        self.cr = correctly_rounded

    def __enter__(self):
        lib().or_set_exp_mode(1 if self.cr else 0)
        return self

    def __exit__(self, *exc):
        lib().or_set_exp_mode(0)


# ---- kernel-level ---------------------------------------------------------
def f16_to_f32(h: int) -> float:
    return lib().or_f16_to_f32(h)


def quantize_i8(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.empty(x.size, dtype=np.int8)
    s = np.zeros(1, dtype=np.float32)
    _check(lib().or_quantize_i8(_ptr(x), x.size, _ptr(q), _ptr(s)), "quantize_i8")
    return q, float(s[0])


def quantize_k(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.empty(x.size, dtype=np.int8)
    s = np.zeros(x.size // 256, dtype=np.float32)
    _check(lib().or_quantize_k(_ptr(x), x.size, _ptr(q), _ptr(s)), "quantize_k")
    return q, s


PARTIALS_PER_BLOCK = {TQ1_0: 1, TQ2_0: 1, Q4_K: 16, Q6_K: 4}


def block_partials(ggml_type: int, q: np.ndarray, w: np.ndarray, n_rows: int, n_cols: int):
    q = np.ascontiguousarray(q, dtype=np.int8)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    out = np.empty(n_rows * (n_cols // 256) * PARTIALS_PER_BLOCK[ggml_type], dtype=np.int32)
    _check(lib().or_block_partials(ggml_type, _ptr(q), _ptr(w), n_rows, n_cols, _ptr(out)),
           "block_partials")
    return out


def gemv_tq_i8(ggml_type, q, scale, w, n_rows, n_cols):
    q = np.ascontiguousarray(q, dtype=np.int8)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    out = np.empty(n_rows, dtype=np.float32)
    _check(lib().or_gemv_tq_i8(ggml_type, _ptr(q), scale, _ptr(w), n_rows, n_cols, _ptr(out)),
           "gemv_tq_i8")
    return out


def gemv(ggml_type, x, w, n_rows, n_cols):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w).view(np.uint8)
    out = np.empty(n_rows, dtype=np.float32)
    _check(lib().or_gemv(ggml_type, _ptr(x), _ptr(w), n_rows, n_cols, _ptr(out)), "gemv")
    return out


def dequant_row(ggml_type, row, n):
    row = np.ascontiguousarray(row).view(np.uint8)
    out = np.empty(n, dtype=np.float32)
    _check(lib().or_dequant_row(ggml_type, _ptr(row), n, _ptr(out)), "dequant_row")
    return out


def tile_attention(q, K, V, nt: int, scale: float):
    """libfoxcuda's tile attention (its production mode) for one query head
    q[hd] over the rows of K, V (P x hd float32)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    V = np.ascontiguousarray(V, dtype=np.float32)
    out = np.empty(q.size, dtype=np.float32)
    _check(lib().or_tile_attention(_ptr(q), _ptr(K), _ptr(V), K.shape[1], q.size, K.shape[0], int(nt),
                                   float(scale), _ptr(out)), "tile_attention")
    return out


def rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().or_rmsnorm(_ptr(out), _ptr(x), _ptr(w), x.size, eps)
    return out


# ---- model-level ----------------------------------------------------------
def _otensor(entry) -> OrTensor:
    tt, ne, data = entry
    return OrTensor(tt, ne[0], ne[1] if len(ne) > 1 else 1, data.ctypes.data)


class OracleModel:
    """The restated forward pass over a rustfox_b200.synth.SyntheticModel."""

    def __init__(self, model):
        c = model.cfg
        self.model = model
        self._keep = [v[2] for v in model.tensors.values()]
        self._layers = (OrLayer * c.n_layer)()
        for l in range(c.n_layer):
            g = lambda k: _otensor(model.tensors[f"blk.{l}.{k}.weight"])
            self._layers[l] = OrLayer(g("attn_norm"), g("attn_q"), g("attn_k"), g("attn_v"),
                                      g("attn_output"), g("ffn_norm"), g("ffn_gate"),
                                      g("ffn_up"), g("ffn_down"))
        info = OrModelInfo(c.n_layer, c.n_embd, c.n_head, c.n_head_kv, c.n_ff,
                           c.head_dim, c.n_vocab, c.rms_eps, c.rope_base)
        self.s = OrModel(info, _otensor(model.tensors["token_embd.weight"]),
                         _otensor(model.tensors["output_norm.weight"]),
                         _otensor(model.tensors["output.weight"]), self._layers)

    def context(self, n_ctx: int, kv_fp16: bool = False, attn_tiles: int = 0) -> "OracleContext":
        """attn_tiles 0: upstream's serial attention; > 0: libfoxcuda's tile
        attention with that tile target (the device's production mode)."""
        return OracleContext(self, n_ctx, kv_fp16, attn_tiles)


class OracleContext:
    def __init__(self, om: OracleModel, n_ctx: int, kv_fp16: bool, attn_tiles: int = 0):
        self.om = om
        self.cfg = om.model.cfg
        self.h = lib().or_ctx_create(C.byref(om.s), n_ctx, 1 if kv_fp16 else 0)
        if not self.h:
            raise MemoryError("oracle context")
        if attn_tiles:
            _check(lib().or_ctx_set_attn_tiles(self.h, int(attn_tiles)), "attention tiles")

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_ctx_destroy(self.h)
            self.h = None

    def reset(self):
        lib().or_ctx_reset(self.h)

    @property
    def pos(self) -> int:
        return lib().or_ctx_pos(self.h)

    def eval(self, tokens, want_hidden: bool = False):
        toks = np.ascontiguousarray(tokens, dtype=np.uint32)
        logits = np.empty(self.cfg.n_vocab, dtype=np.float32)
        hidden = (np.empty((self.cfg.n_layer + 1, self.cfg.n_embd), dtype=np.float32)
                  if want_hidden else None)
        _check(lib().or_eval(self.h, _ptr(toks), toks.size, _ptr(logits),
                             _ptr(hidden) if hidden is not None else None), "eval")
        return (logits, hidden) if want_hidden else logits


class OracleSampler:
    def __init__(self, n_vocab, temperature=0.0, top_k=40, top_p=0.95,
                 repeat_penalty=1.1, repeat_last_n=64, seed=0):
        self.cfg = SamplerConfig(temperature, top_k, top_p, repeat_penalty, repeat_last_n, seed)
        self.h = lib().or_sampler_create(C.byref(self.cfg), n_vocab)

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_sampler_destroy(self.h)
            self.h = None

    def accept(self, tok: int):
        lib().or_sampler_accept(self.h, int(tok))

    def pick(self, logits: np.ndarray) -> int:
        l = np.ascontiguousarray(logits, dtype=np.float32)
        out = np.zeros(1, dtype=np.uint32)
        _check(lib().or_sampler_pick(self.h, _ptr(l), _ptr(out)), "sampler_pick")
        return int(out[0])


def greedy_generate(om: OracleModel, prompt, n_gen: int, n_ctx: int, kv_fp16=False,
                    repeat_penalty=1.1, repeat_last_n=64, attn_tiles=0):
    """The `fox run --temp 0` loop (upstream src/cli.c:333-361) on the oracle:
    eval the prompt, accept it into the sampler history, then pick/accept/eval."""
    ctx = om.context(n_ctx, kv_fp16, attn_tiles)
    smp = OracleSampler(om.model.cfg.n_vocab, temperature=0.0,
                        repeat_penalty=repeat_penalty, repeat_last_n=repeat_last_n)
    logits = ctx.eval(prompt)
    for t in prompt:
        smp.accept(int(t))
    out = []
    for _ in range(n_gen):
        nxt = smp.pick(logits)
        smp.accept(nxt)
        out.append(nxt)
        logits = ctx.eval([nxt])
    return np.array(out, dtype=np.uint32)


# ---- the upstream library itself -------------------------------------------
class FoxContextConfig(C.Structure):
    """upstream fox_context_config (include/fox/fox.h:433-437)"""
    _fields_ = [("n_ctx", _u32), ("n_batch", _u32), ("n_threads", C.c_int)]


class RefLib:
    """The upstream sources built by oracle/Makefile (parity or fast build)."""

    def __init__(self, fast: bool = False):
        path = REF_FAST_SO if fast else REF_SO
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing (built from the upstream sources by "
                               "`make -C oracle ref` where they are available)")
        L = C.CDLL(path)
        L.fox_last_error.restype = C.c_char_p
        L.fox_f16_to_f32.restype = _fp
        L.fox_f16_to_f32.argtypes = [C.c_uint16]
        L.fox_f32_to_f16.restype = C.c_uint16
        L.fox_f32_to_f16.argtypes = [_fp]
        L.fox_quantize_activations_i8.argtypes = [_vp, _sz, _vp, _vp]
        for n in ("fox_tq1_dot_i8", "fox_tq2_dot_i8", "fox_tq1_dot_i8_scalar",
                  "fox_tq2_dot_i8_scalar"):
            getattr(L, n).argtypes = [_vp, _vp, _sz, _vp]
        L.fox_threadpool_create.restype = _vp
        L.fox_threadpool_create.argtypes = [C.c_int]
        L.fox_threadpool_destroy.argtypes = [_vp]
        for n in ("fox_gemv_tq1_i8", "fox_gemv_tq2_i8"):
            getattr(L, n).argtypes = [_vp, _vp, _fp, _vp, _sz, _sz, _vp]
        L.fox_gemv.argtypes = [_vp, C.c_int, _vp, _vp, _sz, _sz, _vp]
        L.fox_dequant_row.argtypes = [C.c_int, _vp, _sz, _vp]
        L.fox_rmsnorm.argtypes = [_vp, _vp, _vp, _sz, _fp]
        L.fox_model_open.argtypes = [C.c_char_p, C.c_int, C.c_uint64, C.POINTER(_vp)]
        L.fox_model_close.argtypes = [_vp]
        L.fox_context_create.argtypes = [_vp, C.POINTER(FoxContextConfig), C.POINTER(_vp)]
        L.fox_context_destroy.argtypes = [_vp]
        L.fox_context_reset.argtypes = [_vp]
        L.fox_eval.argtypes = [_vp, _vp, _sz, C.POINTER(C.POINTER(_fp))]
        L.fox_context_last_eval_seconds.restype = C.c_double
        L.fox_context_last_eval_seconds.argtypes = [_vp]
        L.fox_sampler_create.restype = _vp
        L.fox_sampler_create.argtypes = [C.POINTER(SamplerConfig), _sz]
        L.fox_sampler_destroy.argtypes = [_vp]
        L.fox_sampler_accept.argtypes = [_vp, _u32]
        L.fox_sampler_pick.argtypes = [_vp, _vp, _vp]
        L.fox_cpu_count_online.restype = C.c_int
        self.L = L

    def err(self) -> str:
        return self.L.fox_last_error().decode()

    def gemv(self, ggml_type, x, w, n_rows, n_cols, tp=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w).view(np.uint8)
        out = np.empty(n_rows, dtype=np.float32)
        st = self.L.fox_gemv(tp, ggml_type, _ptr(x), _ptr(w), n_rows, n_cols, _ptr(out))
        if st:
            raise RuntimeError(f"fox_gemv: {st}: {self.err()}")
        return out

    def quantize_i8(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        q = np.empty(x.size, dtype=np.int8)
        s = np.zeros(1, dtype=np.float32)
        st = self.L.fox_quantize_activations_i8(_ptr(x), x.size, _ptr(q), _ptr(s))
        if st:
            raise RuntimeError(f"fox_quantize_activations_i8: {st}")
        return q, float(s[0])

    def gemv_tq_i8(self, ggml_type, q, scale, w, n_rows, n_cols, tp=None):
        fn = self.L.fox_gemv_tq1_i8 if ggml_type == TQ1_0 else self.L.fox_gemv_tq2_i8
        q = np.ascontiguousarray(q, dtype=np.int8)
        w = np.ascontiguousarray(w, dtype=np.uint8)
        out = np.empty(n_rows, dtype=np.float32)
        st = fn(tp, _ptr(q), scale, _ptr(w), n_rows, n_cols, _ptr(out))
        if st:
            raise RuntimeError(f"fox_gemv_tq_i8: {st}: {self.err()}")
        return out

    def dequant_row(self, ggml_type, row, n):
        row = np.ascontiguousarray(row).view(np.uint8)
        out = np.empty(n, dtype=np.float32)
        st = self.L.fox_dequant_row(ggml_type, _ptr(row), n, _ptr(out))
        if st:
            raise RuntimeError(f"fox_dequant_row: {st}: {self.err()}")
        return out

    def open_model(self, path: str):
        h = _vp()
        st = self.L.fox_model_open(path.encode(), 0, 0, C.byref(h))
        if st:
            raise RuntimeError(f"fox_model_open: {st}: {self.err()}")
        return h

    def context(self, model, n_ctx, n_batch=32, n_threads=0):
        cfg = FoxContextConfig(n_ctx, n_batch, n_threads)
        h = _vp()
        st = self.L.fox_context_create(model, C.byref(cfg), C.byref(h))
        if st:
            raise RuntimeError(f"fox_context_create: {st}: {self.err()}")
        return h

    def eval(self, ctx, tokens, n_vocab):
        toks = np.ascontiguousarray(tokens, dtype=np.uint32)
        lp = C.POINTER(_fp)()
        st = self.L.fox_eval(ctx, _ptr(toks), toks.size, C.byref(lp))
        if st:
            raise RuntimeError(f"fox_eval: {st}: {self.err()}")
        return np.ctypeslib.as_array(lp, shape=(n_vocab,)).copy()

    def greedy_generate(self, path, prompt, n_gen, n_ctx, n_vocab, n_threads=0):
        """`fox run --temp 0` on token ids (upstream src/cli.c:333-361)."""
        m = self.open_model(path)
        ctx = self.context(m, n_ctx, 32, n_threads)
        scfg = SamplerConfig(0.0, 40, 0.95, 1.1, 64, 0)
        smp = self.L.fox_sampler_create(C.byref(scfg), n_vocab)
        try:
            logits = self.eval(ctx, prompt, n_vocab)
            first_logits = logits.copy()
            for t in prompt:
                self.L.fox_sampler_accept(smp, int(t))
            out = []
            for _ in range(n_gen):
                o = np.zeros(1, dtype=np.uint32)
                lg = np.ascontiguousarray(logits, dtype=np.float32)
                self.L.fox_sampler_pick(smp, _ptr(lg), _ptr(o))
                nxt = int(o[0])
                self.L.fox_sampler_accept(smp, nxt)
                out.append(nxt)
                logits = self.eval(ctx, [nxt], n_vocab)
            return np.array(out, dtype=np.uint32), first_logits
        finally:
            self.L.fox_sampler_destroy(smp)
            self.L.fox_context_destroy(ctx)
            self.L.fox_model_close(m)
