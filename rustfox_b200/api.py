"""Python host side of libfoxcuda, mirroring upstream RustFox's fox.h API.

The names, argument meaning and error behaviour follow include/fox/fox.h:
  fox_gemv / fox_gemv_tq{1,2}_i8 / fox_quantize_activations_i8 / fox_dequant_row
    -> gemv / gemv_tq1_i8 / gemv_tq2_i8 / quantize_activations_i8 / dequant_row
       (device tensors in, device tensors out)
  fox_model_open / fox_context_create / fox_eval / fox_sampler_*
    -> Model / Context / Sampler (host arrays in and out)
Errors surface as FoxError carrying upstream's fox_status number and the
library's last-error message; there is no CPU fallback: without the CUDA
library the import fails.

torch is used only for device memory and the current CUDA stream.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import formats as F

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libfoxcuda.so")

OK, ERR_ARG, ERR_IO, ERR_NOMEM, ERR_FORMAT, ERR_UNSUPPORTED, ERR_NOTFOUND, ERR_INTERNAL = range(8)
STATUS_NAMES = ["ok", "invalid argument", "io error", "out of memory", "bad format",
                "unsupported", "not found", "internal error"]  # upstream src/log.c:87-100

ROLE = {"token_embd": 0, "output_norm": 1, "output": 2, "attn_norm": 3, "attn_q": 4,
        "attn_k": 5, "attn_v": 6, "attn_output": 7, "ffn_norm": 8, "ffn_gate": 9,
        "ffn_up": 10, "ffn_down": 11}
KV_F16, KV_F32 = 0, 1


class FoxError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES[status] if 0 <= status < 8 else status}: {message}")
        self.status = status
        self.message = message


class ModelInfo(C.Structure):
    _fields_ = [("n_layer", C.c_uint32), ("n_embd", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("n_ff", C.c_uint32), ("head_dim", C.c_uint32),
                ("n_vocab", C.c_uint32), ("rms_eps", C.c_float), ("rope_freq_base", C.c_float)]


class ContextConfig(C.Structure):
    _fields_ = [("n_ctx", C.c_uint32), ("kv_type", C.c_int), ("attn_exact", C.c_int)]


class SamplerConfig(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float),
                ("repeat_penalty", C.c_float), ("repeat_last_n", C.c_uint32),
                ("seed", C.c_uint64)]


_vp, _sz, _st = C.c_void_p, C.c_size_t, C.c_int
_PROTOS = {
    "foxcuda_last_error": (C.c_char_p, []),
    "foxcuda_version": (C.c_char_p, []),
    "foxcuda_init": (_st, [C.c_int]),
    "foxcuda_quantize_activations_i8": (_st, [_vp, _sz, _vp, _vp, _vp]),
    "foxcuda_expf_range": (_st, [C.c_uint32, _sz, _vp, _vp]),
    "foxcuda_gemv_tq1_i8": (_st, [_vp, _vp, _vp, _sz, _sz, _vp, _vp]),
    "foxcuda_gemv_tq2_i8": (_st, [_vp, _vp, _vp, _sz, _sz, _vp, _vp]),
    "foxcuda_gemm_tq_i8": (_st, [C.c_int, _vp, _vp, _sz, _vp, _sz, _sz, _vp, _vp]),
    "foxcuda_gemm_tq2_i8_packed": (_st, [_vp, _vp, _sz, _vp, _sz, _sz, _vp, _vp]),
    "foxcuda_gemm_tq2_i8_split": (_st, [_vp, _vp, _sz, _vp, _sz, _sz, _vp, _vp, _vp]),
    "foxcuda_gemm_kq_i8": (_st, [C.c_int, _vp, _vp, _sz, _vp, _sz, _sz, _vp, _vp]),
    "foxcuda_gemm_kq_i8_packed": (_st, [C.c_int, _vp, _vp, _sz, _vp, _sz, _sz, _vp, _vp]),
    "foxcuda_kernel_errors": (_st, [_vp]),
    "foxcuda_gemv": (_st, [C.c_int, _vp, _vp, _sz, _sz, _vp, _vp]),
    "foxcuda_gemv_noalloc": (_st, [C.c_int, _vp, _vp, _sz, _sz, _vp, _vp]),
    "foxcuda_attn_tile_target": (C.c_int, [C.c_int, C.c_uint32]),
    "foxcuda_attention": (_st, [_vp, _vp, _vp, C.c_int, C.c_uint32, C.c_uint32, C.c_uint32,
                                C.c_uint32, C.c_uint32, C.c_int, _vp, _vp]),
    "foxcuda_dequant_row": (_st, [C.c_int, _vp, _sz, _vp, _vp]),
    "foxcuda_block_partials": (_st, [C.c_int, _vp, _vp, _sz, _sz, _vp, _vp]),
    "foxcuda_packed_bytes": (_sz, [C.c_int, _sz, _sz]),
    "foxcuda_pack": (_st, [C.c_int, _vp, _sz, _sz, _vp, _vp]),
    "foxcuda_gemv_packed": (_st, [C.c_int, _vp, _vp, _sz, _sz, _vp, _vp]),
    "foxcuda_model_create": (_st, [C.POINTER(ModelInfo), C.c_int, C.POINTER(_vp)]),
    "foxcuda_model_upload": (_st, [_vp, C.c_int, C.c_uint32, C.c_int, C.c_uint64, C.c_uint64,
                                   _vp, _sz]),
    "foxcuda_model_upload_synthetic": (_st, [_vp, C.c_int, C.c_uint32, C.c_int, C.c_uint64, C.c_uint64,
                                             C.c_uint64, C.c_float]),
    "foxcuda_model_finalize": (_st, [_vp]),
    "foxcuda_model_destroy": (None, [_vp]),
    "foxcuda_model_device_bytes": (C.c_uint64, [_vp]),
    "foxcuda_model_get_info": (_st, [_vp, C.POINTER(ModelInfo)]),
    "foxcuda_model_save_image": (_st, [_vp, C.c_char_p]),
    "foxcuda_model_open_image": (_st, [C.c_char_p, C.c_int, C.POINTER(_vp)]),
    "foxcuda_context_create": (_st, [_vp, C.POINTER(ContextConfig), C.POINTER(_vp)]),
    "foxcuda_context_create_paged": (_st, [_vp, C.POINTER(ContextConfig), _vp, C.POINTER(_vp)]),
    "foxcuda_kv_pool_create": (_st, [_vp, C.c_uint32, C.c_int, C.POINTER(_vp)]),
    "foxcuda_kv_pool_free_pages": (C.c_uint32, [_vp]),
    "foxcuda_kv_pool_destroy": (_st, [_vp]),
    "foxcuda_context_destroy": (None, [_vp]),
    "foxcuda_context_reset": (None, [_vp]),
    "foxcuda_context_position": (C.c_uint32, [_vp]),
    "foxcuda_context_last_eval_seconds": (C.c_double, [_vp]),
    "foxcuda_eval": (_st, [_vp, _vp, _sz, _vp]),
    "foxcuda_context_set_trace": (_st, [_vp, C.c_int]),
    "foxcuda_context_set_prefill": (_st, [_vp, C.c_int]),
    "foxcuda_eval_all": (_st, [_vp, _vp, _sz, _vp]),
    "foxcuda_context_rewind": (_st, [_vp, C.c_uint32]),
    "foxcuda_context_hidden": (_st, [_vp, C.c_uint32, _vp]),
    "foxcuda_sampler_create": (_st, [_vp, C.POINTER(SamplerConfig), C.POINTER(_vp)]),
    "foxcuda_sampler_destroy": (None, [_vp]),
    "foxcuda_sampler_accept": (_st, [_vp, C.c_uint32]),
    "foxcuda_sampler_pick": (_st, [_vp, _vp]),
    "foxcuda_decode": (_st, [_vp, _vp, C.c_uint32, _vp]),
    "foxcuda_generate": (_st, [_vp, _vp, C.c_uint32, _sz, _vp]),
    "foxcuda_batch_create": (_st, [_vp, _sz, C.POINTER(_vp)]),
    "foxcuda_batch_destroy": (None, [_vp]),
    "foxcuda_batch_step": (_st, [_vp, _vp, _vp]),
    "foxcuda_batch_generate": (_st, [_vp, _vp, _vp, _sz, _vp]),
    "foxcuda_batch_last_seconds": (C.c_double, [_vp]),
    "foxcuda_batch_profile": (_st, [_vp, _vp, _vp, _vp, C.c_int, C.POINTER(C.c_int)]),
    "foxcuda_context_fill_kv": (_st, [_vp, C.c_uint32, C.c_uint64]),
    "foxcuda_context_profile": (_st, [_vp, _vp, C.c_uint32, _vp, _vp, C.c_int,
                                      C.POINTER(C.c_int)]),
    "foxcuda_context_bench_kernel": (_st, [_vp, C.c_int, C.c_int, C.POINTER(C.c_double),
                                           C.POINTER(C.c_uint64)]),
    "foxcuda_model_create_tp": (_st, [C.POINTER(ModelInfo), C.c_int, C.c_int, C.c_int,
                                      C.POINTER(_vp)]),
    "foxcuda_tp_info": (_st, [_vp, _vp]),
    "foxcuda_context_stream": (_vp, [_vp]),
    "foxcuda_tp_embed": (_st, [_vp, C.c_int64]),
    "foxcuda_tp_attention": (_st, [_vp, C.c_uint32]),
    "foxcuda_tp_amax": (_st, [_vp, C.c_int, _vp]),
    "foxcuda_tp_terms": (_st, [_vp, C.c_uint32, C.c_int, _vp, _vp, C.c_uint32]),
    "foxcuda_tp_fold": (_st, [_vp, C.c_uint32, C.c_int, _vp, C.c_uint32, _vp]),
    "foxcuda_tp_ffn": (_st, [_vp, C.c_uint32]),
    "foxcuda_tp_head": (_st, [_vp, _vp]),
    "foxcuda_tp_pick": (_st, [_vp, _vp]),
    "foxcuda_tp_advance": (_st, [_vp]),
    "foxcuda_tp_tokens": (_st, [_vp, C.c_uint32, _sz, _vp]),
    "foxcuda_tp_set_penalty": (_st, [_vp, C.c_float, C.c_uint32]),
    "foxcuda_tp_p2p_export": (_st, [_vp, _vp]),
    "foxcuda_tp_p2p_open": (_st, [_vp, _vp]),
    "foxcuda_tp_p2p_clear": (_st, [_vp]),
    "foxcuda_tp_p2p_row": (_st, [_vp, C.c_uint32, C.c_int]),
    "foxcuda_tp_p2p_pick": (_st, [_vp]),
    "foxcuda_tp_p2p_mode": (_st, [_vp, C.c_int]),
    "foxcuda_tp_feed": (_st, [_vp, C.c_uint32]),
    "foxcuda_tp_p2p_open_local": (_st, [_vp, _vp]),
    "foxcuda_context_logits": (_st, [_vp, _vp, _sz]),
    "foxcuda_context_sync_position": (_st, [_vp]),
}

KIND_NAMES = ["embed", "qkv", "attention", "o", "gate_up", "down", "advance", "head", "pick"]

_lib = None


def lib() -> C.CDLL:
    """The in-tree libfoxcuda.so. Raises when it is missing: there is no
    fallback implementation."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing; build it with "
                              "`python -m rustfox_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _PROTOS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().foxcuda_last_error().decode()


def _check(st: int):
    if st != OK:
        raise FoxError(st, last_error())


def _stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dp(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


# ---- kernel level (torch CUDA tensors) ------------------------------------
def expf_range(first_bits: int, n: int, out=None):
    """The device's e^x (upstream's expf) of the n floats with consecutive bit
    patterns from first_bits, as a float32 CUDA tensor."""
    import torch
    if out is None:
        out = torch.empty(n, dtype=torch.float32, device="cuda")
    _check(lib().foxcuda_expf_range(int(first_bits), int(n), _dp(out), _stream()))
    return out


def quantize_activations_i8(x):
    """upstream fox_quantize_activations_i8 (src/gemv.c:11-42)."""
    import torch
    q = torch.empty(x.numel(), dtype=torch.int8, device=x.device)
    scale = torch.empty(1, dtype=torch.float32, device=x.device)
    _check(lib().foxcuda_quantize_activations_i8(_dp(x), x.numel(), _dp(q), _dp(scale), _stream()))
    return q, scale


def gemv(ggml_type: int, x, w, n_rows: int, n_cols: int, out=None):
    """upstream fox_gemv (src/kernels.c:809-872); w in GGUF layout (uint8)."""
    import torch
    if out is None:
        out = torch.empty(n_rows, dtype=torch.float32, device=x.device)
    _check(lib().foxcuda_gemv(ggml_type, _dp(x), _dp(w), n_rows, n_cols, _dp(out), _stream()))
    return out


def gemv_tq1_i8(q, scale, w, n_rows, n_cols, out=None):
    """upstream fox_gemv_tq1_i8 (src/gemv.c:180-185)."""
    import torch
    out = torch.empty(n_rows, dtype=torch.float32, device=q.device) if out is None else out
    _check(lib().foxcuda_gemv_tq1_i8(_dp(q), _dp(scale), _dp(w), n_rows, n_cols, _dp(out), _stream()))
    return out


def gemv_tq2_i8(q, scale, w, n_rows, n_cols, out=None):
    """upstream fox_gemv_tq2_i8 (src/gemv.c:187-192)."""
    import torch
    out = torch.empty(n_rows, dtype=torch.float32, device=q.device) if out is None else out
    _check(lib().foxcuda_gemv_tq2_i8(_dp(q), _dp(scale), _dp(w), n_rows, n_cols, _dp(out), _stream()))
    return out


def gemm_tq_i8(ggml_type: int, q, scales, w, n_rows: int, n_cols: int, out=None):
    """The per-token fox_gemv_tq{1,2}_i8 of upstream's forward_batch
    (src/forward.c:188-213) for all rows of q (n_tokens x n_cols int8, one
    scale per token) in one tensor-core pass; out is n_tokens x n_rows."""
    import torch
    n_tok = q.shape[0]
    out = torch.empty(n_tok, n_rows, dtype=torch.float32, device=q.device) if out is None else out
    _check(lib().foxcuda_gemm_tq_i8(ggml_type, _dp(q), _dp(scales), n_tok, _dp(w), n_rows, n_cols,
                                    _dp(out), _stream()))
    return out


def gemm_tq2_i8_packed(q, scales, packed, n_rows: int, n_cols: int, out=None):
    """gemm_tq_i8 on TQ2_0 weights already packed by pack()."""
    import torch
    n_tok = q.shape[0]
    out = torch.empty(n_tok, n_rows, dtype=torch.float32, device=q.device) if out is None else out
    _check(lib().foxcuda_gemm_tq2_i8_packed(_dp(q), _dp(scales), n_tok, _dp(packed), n_rows, n_cols,
                                            _dp(out), _stream()))
    return out


def gemm_kq_i8(ggml_type: int, q, scales, w, n_rows: int, n_cols: int, out=None):
    """The per-token K-quant GEMV (upstream gemv_qk_i8, src/kernels.c:571-805)
    for all rows of q (n_tokens x n_cols int8, per-256-block scales
    n_tokens x n_cols/256) in one tensor-core pass; Q4_K or Q6_K GGUF rows."""
    import torch
    n_tok = q.shape[0]
    out = torch.empty(n_tok, n_rows, dtype=torch.float32, device=q.device) if out is None else out
    _check(lib().foxcuda_gemm_kq_i8(ggml_type, _dp(q), _dp(scales), n_tok, _dp(w), n_rows, n_cols,
                                    _dp(out), _stream()))
    return out


def gemm_kq_i8_packed(ggml_type: int, q, scales, packed, n_rows: int, n_cols: int, out=None):
    """gemm_kq_i8 on Q4_K / Q6_K weights already packed by pack()."""
    import torch
    n_tok = q.shape[0]
    out = torch.empty(n_tok, n_rows, dtype=torch.float32, device=q.device) if out is None else out
    _check(lib().foxcuda_gemm_kq_i8_packed(ggml_type, _dp(q), _dp(scales), n_tok, _dp(packed), n_rows,
                                           n_cols, _dp(out), _stream()))
    return out


def gemm_tq2_i8_split(q, scales, packed, n_rows: int, n_cols: int, terms=None, out=None):
    """gemm_tq2_i8_packed with each row's blocks split over CTAs (few tokens);
    terms: device scratch of n_tokens * n_rows * n_cols/256 floats."""
    import torch
    n_tok = q.shape[0]
    if terms is None:
        terms = torch.empty(n_tok * n_rows * (n_cols // 256), dtype=torch.float32, device=q.device)
    out = torch.empty(n_tok, n_rows, dtype=torch.float32, device=q.device) if out is None else out
    _check(lib().foxcuda_gemm_tq2_i8_split(_dp(q), _dp(scales), n_tok, _dp(packed), n_rows, n_cols,
                                           _dp(terms), _dp(out), _stream()))
    return out


def dequant_row(ggml_type: int, row, n: int, out=None):
    """upstream fox_dequant_row (src/kernels.c:874-941)."""
    import torch
    out = torch.empty(n, dtype=torch.float32, device=row.device) if out is None else out
    _check(lib().foxcuda_dequant_row(ggml_type, _dp(row), n, _dp(out), _stream()))
    return out


PARTIALS_PER_BLOCK = {F.TQ1_0: 1, F.TQ2_0: 1, F.Q4_K: 16, F.Q6_K: 4}


def block_partials(ggml_type: int, q, w, n_rows: int, n_cols: int):
    import torch
    out = torch.empty(n_rows * (n_cols // 256) * PARTIALS_PER_BLOCK[ggml_type],
                      dtype=torch.int32, device=q.device)
    _check(lib().foxcuda_block_partials(ggml_type, _dp(q), _dp(w), n_rows, n_cols, _dp(out),
                                        _stream()))
    return out


def pack(ggml_type: int, w, n_rows: int, n_cols: int):
    import torch
    n = lib().foxcuda_packed_bytes(ggml_type, n_rows, n_cols)
    if n == 0:
        raise FoxError(ERR_UNSUPPORTED, f"no packed layout for type {ggml_type}")
    out = torch.empty(n, dtype=torch.uint8, device=w.device)
    _check(lib().foxcuda_pack(ggml_type, _dp(w), n_rows, n_cols, _dp(out), _stream()))
    return out


def gemv_packed(ggml_type: int, x, packed, n_rows: int, n_cols: int, out=None):
    import torch
    out = torch.empty(n_rows, dtype=torch.float32, device=x.device) if out is None else out
    _check(lib().foxcuda_gemv_packed(ggml_type, _dp(x), _dp(packed), n_rows, n_cols, _dp(out),
                                     _stream()))
    return out


# ---- model level (host arrays) --------------------------------------------
class Model:
    """Weights resident in HBM (upstream fox_model_open, src/model.c:146-303)."""

    def __init__(self, info: dict, tensors, device: int = 0, tp_rank: int = 0, tp_size: int = 1):
        """tensors: iterable of (name, ggml_type, ne tuple, host array). With
        tp_size > 1 this is tensor-parallel shard tp_rank: every tensor is
        uploaded whole and the library keeps this shard's part."""
        self.info = dict(info)
        self.tp_rank, self.tp_size = tp_rank, tp_size
        mi = ModelInfo(*(int(info[k]) for k in ("n_layer", "n_embd", "n_head", "n_head_kv",
                                                "n_ff", "head_dim", "n_vocab")),
                       float(info["rms_eps"]), float(info["rope_freq_base"]))
        h = C.c_void_p()
        _check(lib().foxcuda_model_create_tp(C.byref(mi), device, tp_rank, tp_size, C.byref(h)))
        self.h = h
        self.device = device
        try:
            for name, tt, ne, data in tensors:
                role, layer = _role_of(name)
                if role is None:
                    continue
                arr = np.ascontiguousarray(data)
                _check(lib().foxcuda_model_upload(self.h, role, layer, tt, ne[0],
                                                  ne[1] if len(ne) > 1 else 1,
                                                  arr.ctypes.data_as(C.c_void_p), arr.nbytes))
            _check(lib().foxcuda_model_finalize(self.h))
        except Exception:
            self.close()
            raise

    @classmethod
    def from_synthetic(cls, model, device: int = 0, tp_rank: int = 0, tp_size: int = 1) -> "Model":
        c = model.cfg
        info = dict(n_layer=c.n_layer, n_embd=c.n_embd, n_head=c.n_head, n_head_kv=c.n_head_kv,
                    n_ff=c.n_ff, head_dim=c.head_dim, n_vocab=c.n_vocab, rms_eps=c.rms_eps,
                    rope_freq_base=c.rope_base)
        return cls(info, ((n, tt, ne, d) for n, (tt, ne, d) in model.tensors.items()), device,
                   tp_rank, tp_size)

    @classmethod
    def from_synthetic_device(cls, cfg, device: int = 0, tp_rank: int = 0, tp_size: int = 1) -> "Model":
        """A synthetic model of config `cfg` (rustfox_b200.synth) whose weights
        are generated on the device (foxcuda_model_upload_synthetic): the same
        shapes, types and distributions as synth.generate, another stream of
        values, and no host-side generation. For benchmark shapes too large
        to generate on the host (the 27B config)."""
        from . import synth
        info = dict(n_layer=cfg.n_layer, n_embd=cfg.n_embd, n_head=cfg.n_head, n_head_kv=cfg.n_head_kv,
                    n_ff=cfg.n_ff, head_dim=cfg.head_dim, n_vocab=cfg.n_vocab, rms_eps=cfg.rms_eps,
                    rope_freq_base=cfg.rope_base)
        self = cls.__new__(cls)
        self.info, self.device, self.tp_rank, self.tp_size = dict(info), device, tp_rank, tp_size
        mi = ModelInfo(*(int(info[k]) for k in ("n_layer", "n_embd", "n_head", "n_head_kv", "n_ff",
                                                "head_dim", "n_vocab")),
                       float(info["rms_eps"]), float(info["rope_freq_base"]))
        h = C.c_void_p()
        _check(lib().foxcuda_model_create_tp(C.byref(mi), device, tp_rank, tp_size, C.byref(h)))
        self.h = h
        ones = np.ones(cfg.n_embd, dtype=np.float32)
        try:
            for i, (name, tt, ne, sigma) in enumerate(synth.tensor_specs(cfg)):
                role, layer = _role_of(name)
                ne1 = ne[1] if len(ne) > 1 else 1
                if tt == F.F32:
                    _check(lib().foxcuda_model_upload(self.h, role, layer, tt, ne[0], ne1,
                                                      ones.ctypes.data_as(C.c_void_p), ones.nbytes))
                else:
                    _check(lib().foxcuda_model_upload_synthetic(self.h, role, layer, tt, ne[0], ne1,
                                                                synth.device_seed(cfg.seed, i), sigma))
            _check(lib().foxcuda_model_finalize(self.h))
        except Exception:
            self.close()
            raise
        return self

    @classmethod
    def from_gguf(cls, path: str, device: int = 0) -> "Model":
        """Reads the llama metadata the way upstream's loader does
        (src/model.c:188-237): head_dim from attention.key_length, else
        n_embd / n_head; n_vocab from token_embd rows."""
        g = F.read_gguf(path)
        md = g.metadata
        arch = md.get("general.architecture") or "llama"
        get = lambda k, d=None: md.get(f"{arch}.{k}", d)
        n_embd, n_head = int(get("embedding_length")), int(get("attention.head_count"))
        info = dict(n_layer=int(get("block_count")), n_embd=n_embd, n_head=n_head,
                    n_head_kv=int(get("attention.head_count_kv", n_head)),
                    n_ff=int(get("feed_forward_length")),
                    head_dim=int(get("attention.key_length", 0) or n_embd // n_head),
                    n_vocab=g.tensors["token_embd.weight"].ne[1],
                    rms_eps=float(get("attention.layer_norm_rms_epsilon", 1e-5)),
                    rope_freq_base=float(get("rope.freq_base", 10000.0)))
        return cls(info, ((t.name, t.ggml_type, t.ne, g.tensor_bytes(t.name))
                          for t in g.tensors.values()), device)

    def save_image(self, path: str) -> None:
        """Writes this model's HBM layout to a device image (the device-side
        counterpart of upstream's fox_repack_gguf, src/repack.c:170-315)."""
        _check(lib().foxcuda_model_save_image(self.h, os.fsencode(path)))

    @classmethod
    def open_image(cls, path: str, device: int = 0) -> "Model":
        """A model read from a device image onto `device`: one sequential
        read into HBM, no GGUF parse and no packing."""
        h = C.c_void_p()
        _check(lib().foxcuda_model_open_image(os.fsencode(path), device, C.byref(h)))
        self = cls.__new__(cls)
        self.h = h
        self.device = device
        mi = ModelInfo()
        _check(lib().foxcuda_model_get_info(self.h, C.byref(mi)))
        self.info = {name: getattr(mi, name) for name, _ in ModelInfo._fields_}
        from .tp import shape  # tp.py builds on this module
        s = shape(self)
        self.tp_rank, self.tp_size = int(s.tp_rank), int(s.tp_size)
        return self

    @property
    def device_bytes(self) -> int:
        return lib().foxcuda_model_device_bytes(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().foxcuda_model_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    @property
    def attn_tiles(self) -> int:
        """The tile target of this model's tile attention (its production
        mode): foxcuda_attn_tile_target for its device and all its KV heads."""
        return int(lib().foxcuda_attn_tile_target(self.device, int(self.info["n_head_kv"])))

    def context(self, n_ctx: int, kv: str = "f16", attn_exact: bool = False, pool: "KvPool" = None) -> "Context":
        """A decode context; with `pool` its K/V cache is paged from that pool."""
        return Context(self, n_ctx, kv, attn_exact, pool)

    def kv_pool(self, n_pages: int, kv: str = "f16") -> "KvPool":
        return KvPool(self, n_pages, kv)


KV_PAGE = 64  # positions per page (FOXCUDA_KV_PAGE)


class KvPool:
    """A pool of K/V pages shared by paged contexts of one model
    (foxcuda_kv_pool_*): n_pages pages per layer of KV_PAGE positions."""

    def __init__(self, model: "Model", n_pages: int, kv: str = "f16"):
        self.model = model
        h = C.c_void_p()
        _check(lib().foxcuda_kv_pool_create(model.h, int(n_pages), KV_F16 if kv == "f16" else KV_F32,
                                            C.byref(h)))
        self.h = h

    @property
    def free_pages(self) -> int:
        return int(lib().foxcuda_kv_pool_free_pages(self.h))

    def close(self):
        if getattr(self, "h", None):
            _check(lib().foxcuda_kv_pool_destroy(self.h))
            self.h = None


def _role_of(name: str):
    if not name.endswith(".weight"):
        return None, 0
    base = name[:-7]
    if base.startswith("blk."):
        _, l, r = base.split(".", 2)
        return ROLE.get(r), int(l)
    return ROLE.get(base), 0


class Context:
    """upstream fox_context (src/forward.c:9-165): KV cache, scratch, position."""

    def __init__(self, model: Model, n_ctx: int, kv: str = "f16", attn_exact: bool = False,
                 pool: "KvPool" = None):
        """kv: "f16" (default) or "f32" cache; attn_exact: attention in
        upstream's serial operation order (the bit-exact parity mode); pool:
        page the cache from a KvPool."""
        self.model = model
        self.pool = pool
        self.n_vocab = int(model.info["n_vocab"])
        self.n_embd = int(model.info["n_embd"])
        cfg = ContextConfig(n_ctx, KV_F16 if kv == "f16" else KV_F32, 1 if attn_exact else 0)
        h = C.c_void_p()
        if pool is None:
            _check(lib().foxcuda_context_create(model.h, C.byref(cfg), C.byref(h)))
        else:
            _check(lib().foxcuda_context_create_paged(model.h, C.byref(cfg), pool.h, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().foxcuda_context_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def reset(self):
        lib().foxcuda_context_reset(self.h)

    @property
    def pos(self) -> int:
        return lib().foxcuda_context_position(self.h)

    @property
    def last_eval_seconds(self) -> float:
        return lib().foxcuda_context_last_eval_seconds(self.h)

    def set_trace(self, on: bool = True):
        _check(lib().foxcuda_context_set_trace(self.h, 1 if on else 0))

    def fill_kv(self, n_pos: int, seed: int = 1):
        """Seeded N(0, 1) K/V at positions [0, n_pos) and the position set to
        n_pos: a benchmark stand-in for a long prompt."""
        _check(lib().foxcuda_context_fill_kv(self.h, n_pos, seed))

    def set_prefill(self, chunks: bool = True):
        """Prompts of several tokens in chunks through the tensor-core pass
        (True) or one decode step per token (False, the default)."""
        _check(lib().foxcuda_context_set_prefill(self.h, 1 if chunks else 0))

    def eval(self, tokens, want_logits: bool = True):
        """upstream fox_eval: logits (n_vocab, host) of the last token."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self.n_vocab, dtype=np.float32) if want_logits else None
        _check(lib().foxcuda_eval(self.h, t.ctypes.data_as(C.c_void_p), t.size,
                                  out.ctypes.data_as(C.c_void_p) if out is not None else None))
        return out

    def rewind(self, pos: int):
        """Back to an earlier position; the cache from there on is rewritten."""
        _check(lib().foxcuda_context_rewind(self.h, pos))

    def eval_all(self, tokens) -> np.ndarray:
        """The logits of every token, (n, n_vocab): the verification pass of
        speculative decoding."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty((t.size, self.n_vocab), dtype=np.float32)
        _check(lib().foxcuda_eval_all(self.h, t.ctypes.data_as(C.c_void_p), t.size,
                                      out.ctypes.data_as(C.c_void_p)))
        return out

    def hidden(self, layer: int) -> np.ndarray:
        out = np.empty(self.n_embd, dtype=np.float32)
        _check(lib().foxcuda_context_hidden(self.h, layer, out.ctypes.data_as(C.c_void_p)))
        return out

    def sampler(self, **kw) -> "Sampler":
        return Sampler(self, **kw)

    def profile_step(self, token: int, sampler: "Sampler" = None) -> list:
        """One decode step launch by launch: [(kind name, microseconds), ...]."""
        cap = 8192
        us = np.zeros(cap, np.float32)
        kinds = np.zeros(cap, np.int32)
        n = C.c_int()
        _check(lib().foxcuda_context_profile(self.h, sampler.h if sampler else None, int(token),
                                             us.ctypes.data_as(C.c_void_p),
                                             kinds.ctypes.data_as(C.c_void_p), cap, C.byref(n)))
        return [(KIND_NAMES[k], float(t)) for k, t in zip(kinds[:n.value], us[:n.value])]

    def bench_kernel(self, kind: str, reps: int = 64):
        """(microseconds per launch, GGUF weight bytes per launch) of a layer
        GEMV kind ("qkv", "o", "gate_up", "down", "head"); clobbers the
        context's activations (reset before decoding)."""
        us = C.c_double()
        nbytes = C.c_uint64()
        _check(lib().foxcuda_context_bench_kernel(self.h, KIND_NAMES.index(kind), reps,
                                                  C.byref(us), C.byref(nbytes)))
        return us.value, nbytes.value


class Sampler:
    """upstream fox_sampler (src/sample.c), on the device."""

    def __init__(self, ctx: Context, temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.1,
                 repeat_last_n=64, seed=0):
        self.ctx = ctx
        cfg = SamplerConfig(temperature, top_k, top_p, repeat_penalty, repeat_last_n, seed)
        h = C.c_void_p()
        _check(lib().foxcuda_sampler_create(ctx.h, C.byref(cfg), C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().foxcuda_sampler_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def accept(self, token: int):
        _check(lib().foxcuda_sampler_accept(self.h, int(token)))

    def pick(self) -> int:
        out = C.c_uint32()
        _check(lib().foxcuda_sampler_pick(self.h, C.byref(out)))
        return out.value

    def decode(self, token: int) -> int:
        """eval(token) + pick + accept, one CUDA graph (upstream src/cli.c:340-361)."""
        out = C.c_uint32()
        _check(lib().foxcuda_decode(self.ctx.h, self.h, int(token), C.byref(out)))
        return out.value

    def generate(self, token: int, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.uint32)
        _check(lib().foxcuda_generate(self.ctx.h, self.h, int(token), n,
                                      out.ctypes.data_as(C.c_void_p)))
        return out


class Batch:
    """Several contexts of one ternary model decoded together, one pass per
    step (foxcuda_batch_*; no upstream counterpart)."""

    def __init__(self, contexts):
        self.contexts = list(contexts)
        arr = (C.c_void_p * len(self.contexts))(*[c.h.value for c in self.contexts])
        h = C.c_void_p()
        _check(lib().foxcuda_batch_create(arr, len(self.contexts), C.byref(h)))
        self.h = h
        self.n_vocab = self.contexts[0].n_vocab

    def close(self):
        if getattr(self, "h", None):
            lib().foxcuda_batch_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def step(self, tokens=None, want_logits: bool = True):
        """One token per context (host ids, or None for the device tokens);
        the logits (n, n_vocab) of every context."""
        n = len(self.contexts)
        t = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty((n, self.n_vocab), dtype=np.float32) if want_logits else None
        _check(lib().foxcuda_batch_step(self.h, t.ctypes.data_as(C.c_void_p) if t is not None else None,
                                        out.ctypes.data_as(C.c_void_p) if out is not None else None))
        return out

    def generate(self, samplers, n_steps: int, first=None) -> np.ndarray:
        """n_steps steps, each context picking with its sampler; (n_steps, n)."""
        n = len(self.contexts)
        arr = (C.c_void_p * n)(*[s.h.value for s in samplers])
        f = None if first is None else np.ascontiguousarray(first, dtype=np.uint32)
        out = np.empty((n_steps, n), dtype=np.uint32)
        _check(lib().foxcuda_batch_generate(self.h, arr, f.ctypes.data_as(C.c_void_p) if f is not None else None,
                                            n_steps, out.ctypes.data_as(C.c_void_p)))
        return out

    @property
    def last_seconds(self) -> float:
        return lib().foxcuda_batch_last_seconds(self.h)

    def profile_step(self, tokens) -> list:
        """One step on host tokens, phase by phase: [(kind name, microseconds), ...]."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        cap = 4096
        us = np.zeros(cap, np.float32)
        kinds = np.zeros(cap, np.int32)
        n = C.c_int()
        _check(lib().foxcuda_batch_profile(self.h, t.ctypes.data_as(C.c_void_p), us.ctypes.data_as(C.c_void_p),
                                           kinds.ctypes.data_as(C.c_void_p), cap, C.byref(n)))
        return [(KIND_NAMES[k], float(v)) for k, v in zip(kinds[:n.value], us[:n.value])]


def greedy_generate(model: Model, prompt, n_gen: int, n_ctx: int, kv: str = "f16",
                    repeat_penalty: float = 1.1, repeat_last_n: int = 64,
                    attn_exact: bool = False, pool: "KvPool" = None):
    """`fox run --temp 0` on token ids (upstream src/cli.c:333-361): eval the
    prompt, accept it, pick, then decode steps on the device."""
    ctx = Context(model, n_ctx, kv, attn_exact, pool)
    smp = Sampler(ctx, temperature=0.0, repeat_penalty=repeat_penalty,
                  repeat_last_n=repeat_last_n)
    ctx.eval(prompt, want_logits=False)
    for t in prompt:
        smp.accept(int(t))
    first = smp.pick()
    smp.accept(first)
    out = [first]
    if n_gen > 1:
        out += list(smp.generate(first, n_gen - 1))
    smp.close()
    ctx.close()
    return np.array(out[:n_gen], dtype=np.uint32)
