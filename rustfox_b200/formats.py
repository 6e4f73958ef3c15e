"""GGUF v3 reading/writing and ggml block encoders (numpy).

The reader hands tensor bytes to the device weight store; the writer and the
encoders build the seeded synthetic models the tests and the bench run on.

Block layouts follow the upstream RustFox decoders they must round-trip with:
  TQ1_0 54 B/256  src/ternary.c:59-93      TQ2_0 66 B/256  src/ternary.c:177-188
  Q8_0  34 B/32   src/kernels.c:98-113     Q4_K 144 B/256  src/kernels.c:246-283
  Q6_K 210 B/256  src/kernels.c:217-244
GGUF container: upstream src/gguf.c:348-466 (v2/v3, general.alignment).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

# ggml type ids (upstream include/fox/fox.h:203-213)
F32, F16, Q8_0, Q4_K, Q6_K, TQ1_0, TQ2_0 = 0, 1, 8, 12, 14, 34, 35
TYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K",
              TQ1_0: "TQ1_0", TQ2_0: "TQ2_0"}
# (elements per block, bytes per block), upstream src/gguf.c:160-195
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144),
         Q6_K: (256, 210), TQ1_0: (256, 54), TQ2_0: (256, 66)}


def row_bytes(ggml_type: int, n_cols: int) -> int:
    """Bytes of one row of n_cols elements; 0 if n_cols is ragged
    (upstream src/kernels.c:690-698)."""
    blk, nbytes = BLOCK[ggml_type]
    if n_cols % blk:
        return 0
    return n_cols // blk * nbytes


# --- ternary byte codes ----------------------------------------------------
# A TQ1_0 byte packs 5 trits t0..t4 (t0 most significant) as
# ceil((81 t0 + 27 t1 + 9 t2 + 3 t3 + t4) * 256 / 243); a qh byte packs 4 trits
# as ceil((27 t0 + 9 t1 + 3 t2 + t3) * 256 / 81). Level l decodes as
# ((byte * 3^l mod 256) * 3) >> 8 (upstream src/ternary.c:59-63), which these
# encodings invert exactly (tests check all 243 + 81 codes).
TQ1_ENC5 = np.array([(v * 256 + 242) // 243 for v in range(243)], dtype=np.uint8)
TQ1_ENC4 = np.array([(v * 256 + 80) // 81 for v in range(81)], dtype=np.uint8)
_P3 = np.array([1, 3, 9, 27, 81], dtype=np.uint32)


def tq1_decode_level(code: np.ndarray, level: int) -> np.ndarray:
    """Trit value in {-1,0,1} of each byte at a base-3 level."""
    q = (code.astype(np.uint32) * _P3[level]) & 0xFF
    return ((q * 3) >> 8).astype(np.int8) - 1


def encode_tq1(trits: np.ndarray, d: np.ndarray) -> np.ndarray:
    """trits: (nblocks, 256) int values in {-1,0,1}; d: (nblocks,) float16.
    Returns (nblocks, 54) uint8 blocks."""
    t = (np.asarray(trits, dtype=np.int16) + 1).astype(np.uint16)
    nb = t.shape[0]
    out = np.empty((nb, 54), dtype=np.uint8)
    g1 = t[:, :160].reshape(nb, 5, 32)           # element l*32 + m
    g2 = t[:, 160:240].reshape(nb, 5, 16)        # element 160 + l*16 + m
    g3 = t[:, 240:].reshape(nb, 4, 4)            # element 240 + l*4 + m
    v1 = sum(g1[:, l, :] * (3 ** (4 - l)) for l in range(5))
    v2 = sum(g2[:, l, :] * (3 ** (4 - l)) for l in range(5))
    v3 = sum(g3[:, l, :] * (3 ** (3 - l)) for l in range(4))
    out[:, :32] = TQ1_ENC5[v1]
    out[:, 32:48] = TQ1_ENC5[v2]
    out[:, 48:52] = TQ1_ENC4[v3]
    out[:, 52:54] = np.asarray(d, dtype=np.float16).reshape(nb, 1).view(np.uint8)
    return out


def encode_tq2(trits: np.ndarray, d: np.ndarray) -> np.ndarray:
    """TQ2_0: byte qs[j*32+m] holds element j*128 + l*32 + m in bits 2l..2l+1
    as trit+1. Returns (nblocks, 66) uint8."""
    t = (np.asarray(trits, dtype=np.int16) + 1).astype(np.uint8)
    nb = t.shape[0]
    g = t.reshape(nb, 2, 4, 32)                   # [j][l][m]
    qs = np.zeros((nb, 2, 32), dtype=np.uint8)
    for l in range(4):
        qs |= (g[:, :, l, :] << (2 * l)).astype(np.uint8)
    out = np.empty((nb, 66), dtype=np.uint8)
    out[:, :64] = qs.reshape(nb, 64)
    out[:, 64:66] = np.asarray(d, dtype=np.float16).reshape(nb, 1).view(np.uint8)
    return out


def random_tq1_blocks(rng: np.random.Generator, nblocks: int, d_sigma: float) -> np.ndarray:
    """Uniform ternary weights (p = 1/3 each) packed as TQ1_0. A byte of five
    uniform independent trits is a uniform value in [0, 243), so bytes are drawn
    directly. Block scale = |N(0, d_sigma)| as fp16."""
    out = np.empty((nblocks, 54), dtype=np.uint8)
    out[:, :48] = TQ1_ENC5[rng.integers(0, 243, size=(nblocks, 48), dtype=np.uint16)]
    out[:, 48:52] = TQ1_ENC4[rng.integers(0, 81, size=(nblocks, 4), dtype=np.uint16)]
    d = np.abs(rng.normal(0.0, d_sigma, size=nblocks)).astype(np.float16)
    out[:, 52:54] = d.reshape(nblocks, 1).view(np.uint8)
    return out


def random_tq2_blocks(rng: np.random.Generator, nblocks: int, d_sigma: float) -> np.ndarray:
    """Uniform ternary weights packed as TQ2_0 (2-bit codes 0..2 per trit)."""
    codes = rng.integers(0, 3, size=(nblocks, 64, 4), dtype=np.uint8)
    qs = codes[:, :, 0] | (codes[:, :, 1] << 2) | (codes[:, :, 2] << 4) | (codes[:, :, 3] << 6)
    out = np.empty((nblocks, 66), dtype=np.uint8)
    out[:, :64] = qs
    d = np.abs(rng.normal(0.0, d_sigma, size=nblocks)).astype(np.float16)
    out[:, 64:66] = d.reshape(nblocks, 1).view(np.uint8)
    return out


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest Q8_0 of a float array whose length is a multiple of 32
    (d = amax/127 as fp16). Returns (n/32, 34) uint8."""
    xb = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    amax = np.abs(xb).max(axis=1)
    d = (amax / 127.0).astype(np.float16)
    df = d.astype(np.float32)
    inv = np.where(df > 0, 1.0 / np.where(df > 0, df, 1.0), 0.0).astype(np.float32)
    q = np.clip(np.rint(xb * inv[:, None]), -127, 127).astype(np.int8)
    out = np.empty((xb.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d.reshape(-1, 1).view(np.uint8)
    out[:, 2:] = q.view(np.uint8)
    return out


def random_q8_0_blocks(rng: np.random.Generator, n_elems: int, sigma: float,
                       chunk: int = 1 << 24) -> np.ndarray:
    """Q8_0 of N(0, sigma) values, generated in chunks to bound host memory."""
    out = np.empty((n_elems // 32, 34), dtype=np.uint8)
    done = 0
    while done < n_elems:
        n = min(chunk, n_elems - done)
        out[done // 32:(done + n) // 32] = quantize_q8_0(
            rng.normal(0.0, sigma, size=n).astype(np.float32))
        done += n
    return out


def random_q4_k_blocks(rng: np.random.Generator, nblocks: int, d_sigma: float) -> np.ndarray:
    """Q4_K: fp16 d and dmin = |N(0, d_sigma)|, uniform 6-bit scales/mins (any
    12-byte pattern is valid) and uniform 4-bit quants."""
    out = rng.integers(0, 256, size=(nblocks, 144), dtype=np.uint8)
    d = np.abs(rng.normal(0.0, d_sigma, size=(nblocks, 2))).astype(np.float16)
    out[:, 0:4] = d.view(np.uint8).reshape(nblocks, 4)
    return out


def random_q6_k_blocks(rng: np.random.Generator, nblocks: int, d_sigma: float) -> np.ndarray:
    """Q6_K: uniform 6-bit quants (ql/qh bytes), uniform int8 sub-scales,
    fp16 d = |N(0, d_sigma)| at byte 208."""
    out = rng.integers(0, 256, size=(nblocks, 210), dtype=np.uint8)
    d = np.abs(rng.normal(0.0, d_sigma, size=nblocks)).astype(np.float16)
    out[:, 208:210] = d.reshape(nblocks, 1).view(np.uint8)
    return out


def random_blocks(rng: np.random.Generator, ggml_type: int, n_rows: int, n_cols: int,
                  sigma: float) -> np.ndarray:
    """Seeded random weights of a quantised type as a flat uint8 array laid out
    row-major (GGUF ne1 x ne0)."""
    blk, _ = BLOCK[ggml_type]
    nb = n_rows * (n_cols // blk)
    if ggml_type == TQ1_0:
        b = random_tq1_blocks(rng, nb, sigma)
    elif ggml_type == TQ2_0:
        b = random_tq2_blocks(rng, nb, sigma)
    elif ggml_type == Q8_0:
        b = random_q8_0_blocks(rng, n_rows * n_cols, sigma)
    elif ggml_type == Q4_K:
        b = random_q4_k_blocks(rng, nb, sigma)
    elif ggml_type == Q6_K:
        b = random_q6_k_blocks(rng, nb, sigma)
    else:
        raise ValueError(f"no random generator for type {ggml_type}")
    return b.reshape(-1)


# --- GGUF container --------------------------------------------------------
GGUF_U8, GGUF_I8, GGUF_U16, GGUF_I16, GGUF_U32, GGUF_I32, GGUF_F32, GGUF_BOOL, \
    GGUF_STR, GGUF_ARR, GGUF_U64, GGUF_I64, GGUF_F64 = range(13)
_SCALAR = {GGUF_U8: "<B", GGUF_I8: "<b", GGUF_U16: "<H", GGUF_I16: "<h",
           GGUF_U32: "<I", GGUF_I32: "<i", GGUF_F32: "<f", GGUF_BOOL: "<?",
           GGUF_U64: "<Q", GGUF_I64: "<q", GGUF_F64: "<d"}


@dataclass
class TensorInfo:
    name: str
    ne: tuple
    ggml_type: int
    offset: int          # relative to the data section
    nbytes: int


@dataclass
class GGUFFile:
    path: str
    version: int
    metadata: dict
    tensors: dict = field(default_factory=dict)   # name -> TensorInfo
    data_offset: int = 0
    alignment: int = 32
    _mm: np.memmap | None = None

    def tensor_bytes(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        if self._mm is None:
            self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        start = self.data_offset + t.offset
        return self._mm[start:start + t.nbytes]


def _read_str(buf, pos):
    (n,) = struct.unpack_from("<Q", buf, pos)
    pos += 8
    return bytes(buf[pos:pos + n]).decode("utf-8", "replace"), pos + n


def _read_value(buf, pos, vt):
    if vt == GGUF_STR:
        return _read_str(buf, pos)
    if vt == GGUF_ARR:
        (et, n) = struct.unpack_from("<IQ", buf, pos)
        pos += 12
        vals = []
        for _ in range(n):
            v, pos = _read_value(buf, pos, et)
            vals.append(v)
        return vals, pos
    fmt = _SCALAR[vt]
    (v,) = struct.unpack_from(fmt, buf, pos)
    return v, pos + struct.calcsize(fmt)


def read_gguf(path: str, skip_arrays: bool = True) -> GGUFFile:
    """Parses the header, metadata and tensor table of a GGUF v2/v3 file.
    Array metadata (tokenizer vocab) is skipped unless asked for."""
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    buf = memoryview(mm)
    if bytes(buf[:4]) != b"GGUF":
        raise ValueError(f"{path} is not a GGUF file")
    version, n_t, n_kv = struct.unpack_from("<IQQ", buf, 4)
    if version not in (2, 3):
        raise ValueError(f"GGUF version {version} not supported")
    pos = 24
    meta = {}
    for _ in range(n_kv):
        key, pos = _read_str(buf, pos)
        (vt,) = struct.unpack_from("<I", buf, pos)
        pos += 4
        if vt == GGUF_ARR and skip_arrays:
            (et, n) = struct.unpack_from("<IQ", buf, pos)
            pos += 12
            if et == GGUF_STR:
                for _ in range(n):
                    (ln,) = struct.unpack_from("<Q", buf, pos)
                    pos += 8 + ln
            else:
                pos += n * struct.calcsize(_SCALAR[et])
            meta[key] = None
            continue
        meta[key], pos = _read_value(buf, pos, vt)
    align = int(meta.get("general.alignment", 32))
    f = GGUFFile(path=path, version=version, metadata=meta, alignment=align, _mm=mm)
    for _ in range(n_t):
        name, pos = _read_str(buf, pos)
        (nd,) = struct.unpack_from("<I", buf, pos)
        pos += 4
        ne = struct.unpack_from("<" + "Q" * nd, buf, pos)
        pos += 8 * nd
        ttype, off = struct.unpack_from("<IQ", buf, pos)
        pos += 12
        n_el = int(np.prod(ne))
        blk, nbytes = BLOCK.get(ttype, (1, 0))
        f.tensors[name] = TensorInfo(name, tuple(int(v) for v in ne), ttype, off,
                                     n_el // blk * nbytes)
    f.data_offset = (pos + align - 1) // align * align
    return f


class GGUFWriter:
    """Minimal GGUF v3 writer: metadata then tensors, each at an aligned offset."""

    def __init__(self, path: str, alignment: int = 32):
        self.path = path
        self.alignment = alignment
        self.kv: list[tuple[str, int, object]] = []
        self.tensors: list[tuple[str, tuple, int, object]] = []
        self.add_u32("general.alignment", alignment)

    def add_u32(self, key, v):
        self.kv.append((key, GGUF_U32, int(v)))

    def add_f32(self, key, v):
        self.kv.append((key, GGUF_F32, float(v)))

    def add_str(self, key, v):
        self.kv.append((key, GGUF_STR, str(v)))

    def add_str_array(self, key, values):
        self.kv.append((key, GGUF_ARR, (GGUF_STR, list(values))))

    def add_f32_array(self, key, values):
        self.kv.append((key, GGUF_ARR, (GGUF_F32, np.asarray(values, dtype=np.float32))))

    def add_tensor(self, name, ne, ggml_type, data):
        """ne: (ne0,) or (ne0, ne1); data: anything np.asarray can view as bytes."""
        self.tensors.append((name, tuple(int(v) for v in ne), int(ggml_type), data))

    @staticmethod
    def _str(s: str) -> bytes:
        b = s.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    def _value(self, vt, v) -> bytes:
        if vt == GGUF_STR:
            return self._str(v)
        if vt == GGUF_ARR:
            et, vals = v
            head = struct.pack("<IQ", et, len(vals))
            if et == GGUF_STR:
                return head + b"".join(self._str(s) for s in vals)
            return head + np.asarray(vals).astype(_SCALAR[et]).tobytes()
        return struct.pack(_SCALAR[vt], v)

    def write(self):
        a = self.alignment
        head = [b"GGUF", struct.pack("<IQQ", 3, len(self.tensors), len(self.kv))]
        for key, vt, v in self.kv:
            head += [self._str(key), struct.pack("<I", vt), self._value(vt, v)]
        offset = 0
        blobs = []
        for name, ne, tt, data in self.tensors:
            b = np.ascontiguousarray(np.asarray(data)).view(np.uint8).reshape(-1)
            blk, nbytes = BLOCK[tt]
            want = int(np.prod(ne)) // blk * nbytes
            if b.size != want:
                raise ValueError(f"{name}: {b.size} bytes, type wants {want}")
            head += [self._str(name), struct.pack("<I", len(ne)),
                     struct.pack("<" + "Q" * len(ne), *ne), struct.pack("<IQ", tt, offset)]
            blobs.append((offset, b))
            offset = (offset + b.size + a - 1) // a * a
        header = b"".join(head)
        data_start = (len(header) + a - 1) // a * a
        with open(self.path, "wb") as fh:
            fh.write(header)
            fh.write(b"\0" * (data_start - len(header)))
            pos = 0
            for off, b in blobs:
                if off > pos:
                    fh.write(b"\0" * (off - pos))
                fh.write(memoryview(b))
                pos = off + b.size
