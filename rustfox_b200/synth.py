"""Seeded synthetic Llama-architecture models (the benchmark configurations).

There are no real checkpoints on the machines this runs on, so every model is
random-initialised from a numpy PCG64 stream seeded with the config's seed,
with the shapes, quantisation types and value distributions the benchmark
configurations name:
  TQ1_0/TQ2_0 linear: uniform ternary weights, fp16 block scale |N(0, 0.02)|
  Q4_K/Q6_K: uniform quants and sub-scales, fp16 super-scales |N(0, 0.01)|
  Q8_0 embedding and output head: N(0, 0.02); norm weights 1.0 (F32).

Tensor names and metadata keys are the ones upstream's loader resolves
(upstream src/model.c:51-83, 188-237); head_dim is always written as
llama.attention.key_length because the 4B shape has n_head*head_dim != n_embd.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, replace

import numpy as np

from . import formats as F


@dataclass(frozen=True)
class ModelConfig:
    name: str
    n_layer: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_ff: int
    n_vocab: int
    rope_base: float
    rms_eps: float = 1e-5
    linear_type: int = F.TQ1_0
    attn_v_type: int | None = None
    embd_type: int = F.Q8_0
    output_type: int = F.Q8_0
    ctx_len: int = 4096
    linear_sigma: float = 0.02
    embd_sigma: float = 0.02
    seed: int = 0

    def scaled(self, **kw) -> "ModelConfig":
        return replace(self, **kw)

    def linear_types(self) -> dict:
        t = self.linear_type
        return {"attn_q": t, "attn_k": t, "attn_v": self.attn_v_type or t,
                "attn_output": t, "ffn_gate": t, "ffn_up": t, "ffn_down": t}

    def shapes(self) -> dict:
        """(ne0 = input columns, ne1 = output rows) of each per-layer matrix."""
        nq, nkv = self.n_head * self.head_dim, self.n_head_kv * self.head_dim
        e, f = self.n_embd, self.n_ff
        return {"attn_q": (e, nq), "attn_k": (e, nkv), "attn_v": (e, nkv),
                "attn_output": (nq, e), "ffn_gate": (e, f), "ffn_up": (e, f),
                "ffn_down": (f, e)}

    def weight_bytes(self) -> dict:
        """GGUF bytes per tensor class: the algorithmic weight bytes a decode
        token streams once."""
        per_layer = sum(F.row_bytes(self.linear_types()[k], ne0) * ne1
                        for k, (ne0, ne1) in self.shapes().items())
        return {
            "layers": per_layer * self.n_layer,
            "output": F.row_bytes(self.output_type, self.n_embd) * self.n_vocab,
            "embd_row": F.row_bytes(self.embd_type, self.n_embd),
            "norms": (2 * self.n_layer + 1) * self.n_embd * 4,
        }

    def kv_bytes_per_token(self, pos: int, kv_elem_bytes: int = 2) -> int:
        """K and V read for positions 0..pos plus the write at pos, all layers."""
        row = self.n_head_kv * self.head_dim * kv_elem_bytes
        return 2 * self.n_layer * row * (pos + 1) + 2 * self.n_layer * row


# The five benchmark configurations. The tiny config's FFN is 1536 instead of
# the stated 1408: 1408 = 5.5 * 256 cannot be the K of a 256-block ternary
# ffn_down, which upstream rejects at the first eval (src/gemv.c:82-85).
CONFIGS = {
    "tiny": ModelConfig("tiny", 8, 512, 8, 2, 64, 1536, 32000, 1e4, ctx_len=256),
    "4b": ModelConfig("4b", 36, 2560, 32, 8, 128, 9728, 151936, 1e6, ctx_len=4096),
    "8b": ModelConfig("8b", 32, 4096, 32, 8, 128, 14336, 128256, 5e5,
                      linear_type=F.Q4_K, attn_v_type=F.Q6_K, output_type=F.Q6_K,
                      ctx_len=8192, linear_sigma=0.01),
    "27b": ModelConfig("27b", 62, 5120, 32, 16, 128, 21504, 262144, 1e6,
                       linear_type=F.TQ2_0, ctx_len=2048),
    "8b-tq2": ModelConfig("8b-tq2", 32, 4096, 32, 8, 128, 14336, 128256, 5e5,
                          linear_type=F.TQ2_0, output_type=F.Q6_K, ctx_len=32896),
}


class SyntheticModel:
    """Tensors in GGUF order: name -> (ggml_type, ne tuple, flat array)."""

    def __init__(self, cfg: ModelConfig):
        self.cfg = cfg
        self.tensors: "OrderedDict[str, tuple]" = OrderedDict()

    def metadata(self) -> dict:
        c = self.cfg
        return {
            "general.architecture": "llama", "general.name": f"synthetic-{c.name}",
            "llama.block_count": c.n_layer, "llama.embedding_length": c.n_embd,
            "llama.attention.head_count": c.n_head,
            "llama.attention.head_count_kv": c.n_head_kv,
            "llama.attention.key_length": c.head_dim,
            "llama.feed_forward_length": c.n_ff, "llama.context_length": c.ctx_len,
            "llama.attention.layer_norm_rms_epsilon": c.rms_eps,
            "llama.rope.freq_base": c.rope_base,
        }

    def tensor(self, name: str):
        return self.tensors[name]


def _weights(rng, ggml_type, ne0, ne1, sigma):
    return F.random_blocks(rng, ggml_type, ne1, ne0, sigma)


def tensor_specs(cfg: ModelConfig):
    """(name, ggml_type, ne, sigma) of every tensor in GGUF order; F32 tensors
    are the norm weights (all ones, sigma 0)."""
    e = cfg.n_embd
    yield "token_embd.weight", cfg.embd_type, (e, cfg.n_vocab), cfg.embd_sigma
    yield "output_norm.weight", F.F32, (e,), 0.0
    yield ("output.weight", cfg.output_type, (e, cfg.n_vocab),
           cfg.embd_sigma if cfg.output_type == F.Q8_0 else 0.01)
    types, shapes = cfg.linear_types(), cfg.shapes()
    for l in range(cfg.n_layer):
        yield f"blk.{l}.attn_norm.weight", F.F32, (e,), 0.0
        for k in ("attn_q", "attn_k", "attn_v", "attn_output"):
            yield (f"blk.{l}.{k}.weight", types[k], shapes[k],
                   cfg.linear_sigma if types[k] == cfg.linear_type else 0.01)
        yield f"blk.{l}.ffn_norm.weight", F.F32, (e,), 0.0
        for k in ("ffn_gate", "ffn_up", "ffn_down"):
            yield f"blk.{l}.{k}.weight", types[k], shapes[k], cfg.linear_sigma


def generate(cfg: ModelConfig) -> SyntheticModel:
    """Deterministic in cfg (including cfg.seed)."""
    rng = np.random.Generator(np.random.PCG64(cfg.seed))
    m = SyntheticModel(cfg)
    ones = np.ones(cfg.n_embd, dtype=np.float32)
    for name, tt, ne, sigma in tensor_specs(cfg):
        m.tensors[name] = (tt, ne, ones if tt == F.F32 else _weights(rng, tt, ne[0], ne[1], sigma))
    return m


def _timing_blocks(rng, ggml_type: int, ne0: int, ne1: int, sigma: float) -> np.ndarray:
    """Uniform random bytes in the layout of ggml_type with every scale a
    finite fp16 of size sigma (ternary codes kept in 0..2)."""
    nb = ne1 * (ne0 // F.BLOCK[ggml_type][0])
    if ggml_type == F.Q8_0:
        b = rng.integers(0, 256, size=(nb, 34), dtype=np.uint8)
        b[:, 0:2] = np.full((nb, 1), sigma / 127.0 * 3.0, np.float16).view(np.uint8)
    elif ggml_type == F.TQ2_0:
        b = rng.integers(0, 256, size=(nb, 66), dtype=np.uint8)
        q = b[:, :64]
        q ^= q & (q >> 1) & np.uint8(0x55)  # a code of 3 becomes 2
        b[:, 64:66] = np.full((nb, 1), sigma, np.float16).view(np.uint8)
    else:
        raise ValueError(f"no timing sample for type {ggml_type}")
    return b.reshape(-1)


def timing_sample(cfg: ModelConfig, n_layer: int, seed: int = 0, shared: dict | None = None) -> SyntheticModel:
    """A model with cfg's shapes and types and n_layer layers whose bytes are
    drawn uniformly (valid scales), for timing a CPU decode of a model too
    large to generate quickly: every layer reuses the same tensors, and
    `shared` (a dict, filled on first use) carries the embedding and head
    from one sample to the next. A decode's time does not depend on these
    values; its results are not meant to be compared."""
    c = cfg.scaled(n_layer=n_layer)
    rng = np.random.Generator(np.random.PCG64(seed))
    shared = {} if shared is None else shared
    m = SyntheticModel(c)
    ones = np.ones(c.n_embd, dtype=np.float32)
    for name, tt, ne, sigma in tensor_specs(c):
        if tt == F.F32:
            m.tensors[name] = (tt, ne, ones)
            continue
        key = name if not name.startswith("blk.") else name.split(".", 2)[2]
        if key not in shared:
            shared[key] = _timing_blocks(rng, tt, ne[0], ne[1], sigma)
        m.tensors[name] = (tt, ne, shared[key])
    return m


def device_seed(cfg_seed: int, index: int) -> int:
    """The seed of tensor `index` (GGUF order) of a model generated on the
    device (foxcuda_model_upload_synthetic)."""
    return (((cfg_seed + 1) * 0x9E3779B97F4A7C15) ^ ((index + 1) * 0xD1B54A32D192ED03)) & (2**64 - 1)


def byte_vocab(n_vocab: int) -> list:
    """Byte-level vocabulary: <0x00>..<0xFF> then inert filler entries."""
    toks = [f"<0x{i:02X}>" for i in range(min(256, n_vocab))]
    toks += [f"[t{i}]" for i in range(len(toks), n_vocab)]
    return toks


def write_gguf(model: SyntheticModel, path: str, tokenizer: bool = True) -> str:
    """Writes the model as GGUF v3 (alignment 32). The tokenizer metadata is a
    byte-level vocabulary with no eos id, so decoding never stops early."""
    w = F.GGUFWriter(path)
    for k, v in model.metadata().items():
        if isinstance(v, str):
            w.add_str(k, v)
        elif isinstance(v, float):
            w.add_f32(k, v)
        else:
            w.add_u32(k, v)
    if tokenizer:
        vocab = byte_vocab(model.cfg.n_vocab)
        w.add_str("tokenizer.ggml.model", "llama")
        w.add_str_array("tokenizer.ggml.tokens", vocab)
        w.add_f32_array("tokenizer.ggml.scores",
                        [0.0] * min(256, len(vocab)) + [-1000.0] * max(0, len(vocab) - 256))
    for name, (tt, ne, data) in model.tensors.items():
        w.add_tensor(name, ne, tt, data)
    w.write()
    return path


def random_prompt(cfg: ModelConfig, n: int, seed: int = 1) -> np.ndarray:
    """Uniform random prompt token ids (seeded)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(0, cfg.n_vocab, size=n, dtype=np.uint32)
