"""A numpy restatement of the device-side synthetic weight generator
(rustfox_b200/csrc/synthgen.cuh, foxcuda_model_upload_synthetic), for the
tests: the same counters, the same splitmix64 finalizer, Box-Muller in
double, the same roundings. A model built from these host tensors must hold
the same bytes as one generated on the device.
"""
import numpy as np

from rustfox_b200 import formats as F

U64 = np.uint64
STRIDE = {F.TQ1_0: 64, F.TQ2_0: 80, F.Q8_0: 48, F.Q4_K: 160, F.Q6_K: 224}


def mix(seed: int, i: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = U64(seed) + (i.astype(U64) + U64(1)) * U64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> U64(30))) * U64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> U64(27))) * U64(0x94D049BB133111EB)
        return z ^ (z >> U64(31))


def normal2(seed: int, i: np.ndarray):
    u1 = ((mix(seed, i) >> U64(11)).astype(np.float64) + 1.0) * 2.0**-53
    u2 = (mix(seed, i + U64(1)) >> U64(11)).astype(np.float64) * 2.0**-53
    r, t = np.sqrt(-2.0 * np.log(u1)), 6.283185307179586 * u2
    return r * np.cos(t), r * np.sin(t)


def below(h: np.ndarray, n: int) -> np.ndarray:
    return ((h >> U64(32)) * U64(n)) >> U64(32)


def half_abs(z: np.ndarray, sigma: float) -> np.ndarray:
    return np.abs(z * sigma).astype(np.float32).astype(np.float16).view(np.uint16)


def _put16(out, col, v):
    out[:, col] = (v & 0xFF).astype(np.uint8)
    out[:, col + 1] = (v >> 8).astype(np.uint8)


def blocks(ggml_type: int, n_rows: int, n_cols: int, seed: int, sigma: float) -> np.ndarray:
    """The tensor's bytes, row-major (GGUF ne1 x ne0), as the device writes them."""
    blk, bb = F.BLOCK[ggml_type]
    nb = n_rows * (n_cols // blk)
    sigma = float(np.float32(sigma))  # the entry point takes a float
    base = np.arange(nb, dtype=U64)[:, None] * U64(STRIDE[ggml_type])
    out = np.zeros((nb, bb), dtype=np.uint8)
    if ggml_type == F.TQ1_0:
        v5 = below(mix(seed, base + np.arange(48, dtype=U64)), 243)
        out[:, :48] = ((v5 * U64(256) + U64(242)) // U64(243)).astype(np.uint8)
        v4 = below(mix(seed, base + np.arange(48, 52, dtype=U64)), 81)
        out[:, 48:52] = ((v4 * U64(256) + U64(80)) // U64(81)).astype(np.uint8)
        z0, _ = normal2(seed, base[:, 0] + U64(52))
        _put16(out, 52, half_abs(z0, sigma))
    elif ggml_type == F.TQ2_0:
        c = below(mix(seed, base + np.arange(64, dtype=U64)), 81)
        out[:, :64] = (c % U64(3) | (c // U64(3) % U64(3)) << U64(2) | (c // U64(9) % U64(3)) << U64(4)
                       | (c // U64(27)) << U64(6)).astype(np.uint8)
        z0, _ = normal2(seed, base[:, 0] + U64(64))
        _put16(out, 64, half_abs(z0, sigma))
    elif ggml_type == F.Q8_0:
        z0, z1 = normal2(seed, base + np.arange(0, 32, 2, dtype=U64))
        x = np.empty((nb, 32), dtype=np.float32)
        x[:, 0::2] = (z0 * sigma).astype(np.float32)
        x[:, 1::2] = (z1 * sigma).astype(np.float32)
        amax = np.abs(x).max(axis=1)
        d = (amax / np.float32(127.0)).astype(np.float32).astype(np.float16)
        df = d.astype(np.float32)
        inv = np.where(df > 0, np.float32(1.0) / np.where(df > 0, df, np.float32(1.0)), np.float32(0.0))
        q = np.clip(np.rint((x * inv[:, None].astype(np.float32)).astype(np.float32)), -127, 127)
        _put16(out, 0, d.view(np.uint16))
        out[:, 2:] = q.astype(np.int8).view(np.uint8)
    elif ggml_type == F.Q4_K:
        out[:, 4:144] = (mix(seed, base + np.arange(4, 144, dtype=U64)) >> U64(56)).astype(np.uint8)
        z0, z1 = normal2(seed, base[:, 0] + U64(144))
        _put16(out, 0, half_abs(z0, sigma))
        _put16(out, 2, half_abs(z1, sigma))
    elif ggml_type == F.Q6_K:
        out[:, :208] = (mix(seed, base + np.arange(208, dtype=U64)) >> U64(56)).astype(np.uint8)
        z0, _ = normal2(seed, base[:, 0] + U64(208))
        _put16(out, 208, half_abs(z0, sigma))
    else:
        raise ValueError(f"no device generator for type {ggml_type}")
    return out.reshape(-1)


def tensors(cfg):
    """(name, ggml_type, ne, host array) of the model Model.from_synthetic_device
    builds for cfg, in GGUF order."""
    from rustfox_b200 import synth
    ones = np.ones(cfg.n_embd, dtype=np.float32)
    for i, (name, tt, ne, sigma) in enumerate(synth.tensor_specs(cfg)):
        if tt == F.F32:
            yield name, tt, ne, ones
        else:
            yield name, tt, ne, blocks(tt, ne[1], ne[0], synth.device_seed(cfg.seed, i), sigma)
