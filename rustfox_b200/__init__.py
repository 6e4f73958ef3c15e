"""rustfox_b200: RustFox's per-token forward pass on B200 (sm_100a).

The compute lives in libfoxcuda.so (C ABI, include/foxcuda.h); this package
is its Python host side, mirroring upstream RustFox's fox.h API, plus the GGUF
and synthetic-model helpers.
"""
from . import formats, spec, synth  # noqa: F401
from .api import (FoxError, Model, Context, KvPool, Sampler, Batch, lib, last_error,  # noqa: F401
                  quantize_activations_i8, gemv, gemv_tq1_i8, gemv_tq2_i8, gemm_tq_i8,
                  gemm_tq2_i8_packed, gemm_tq2_i8_split, gemm_kq_i8, gemm_kq_i8_packed,
                  dequant_row, block_partials, pack, gemv_packed, greedy_generate)

__all__ = ["formats", "synth", "FoxError", "Model", "Context", "KvPool", "Sampler", "Batch", "lib", "last_error",
           "quantize_activations_i8", "gemv", "gemv_tq1_i8", "gemv_tq2_i8", "gemm_tq_i8",
           "gemm_tq2_i8_packed", "gemm_tq2_i8_split", "gemm_kq_i8", "gemm_kq_i8_packed", "dequant_row", "block_partials", "pack", "gemv_packed",
           "greedy_generate"]
