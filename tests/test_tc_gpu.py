"""The M-token ternary pass on the tensor cores (tcgen05 kind::i8) against the
oracle, bit for bit.

Upstream's forward_batch runs one fox_gemv_tq{1,2}_i8 per token
(src/forward.c:188-213), each token quantised with its own absmax scale
(src/gemv.c:11-42). foxcuda_gemm_tq_i8 does all tokens in one pass and must
give every token exactly that GEMV's row. The cases cover each token tile
(MMA N = 8, 16, 32, 64), several token tiles, rows that end inside a 128-row
tile, both ternary types, one block per row up to the 84 blocks of the 27B
down projection, and 2-bit codes of 3 (weight 2), which upstream's TQ2_0
decode accepts.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
from rustfox_b200 import formats as F  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

DEV = "cuda:0"


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _u32(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def _tokens(rng, n_tok, cols):
    """n_tok activation vectors, each quantised with its own scale."""
    q = np.empty((n_tok, cols), dtype=np.int8)
    s = np.empty(n_tok, dtype=np.float32)
    for t in range(n_tok):
        q[t], s[t] = O.quantize_i8(rng.normal(0, 1, cols).astype(np.float32))
    return q, s


def _check_rows(got, tt, q, s, w, rows, cols):
    for t in range(q.shape[0]):
        want = O.gemv_tq_i8(tt, q[t], float(s[t]), w, rows, cols)
        bad = np.count_nonzero(_u32(got[t]) != _u32(want))
        assert bad == 0, f"token {t}: {bad} of {rows} rows differ; max |d| {np.abs(got[t] - want).max()}"


CASES = [
    (F.TQ2_0, 200, 768, 9),     # N = 16, the last row tile partial
    (F.TQ1_0, 130, 512, 3),     # N = 8, transcoded to TQ2_0
    (F.TQ2_0, 64, 256, 40),     # N = 64, one block per row
    (F.TQ2_0, 300, 2560, 1),    # a single token
    (F.TQ2_0, 1000, 2560, 33),  # N = 64, the token tile partial
    (F.TQ1_0, 517, 1024, 100),  # two token tiles
    (F.TQ2_0, 2560, 9728, 16),  # the 4B down projection, 38 blocks
    (F.TQ2_0, 256, 21504, 8),   # 84 blocks (the 27B down projection's K)
    (F.TQ2_0, 4096, 2560, 24),  # N = 32, the 4B q projection
]


@pytest.mark.parametrize("tt,rows,cols,n_tok", CASES)
def test_gemm_equals_per_token_gemv(tt, rows, cols, n_tok):
    rng = np.random.default_rng(rows * 3 + cols + n_tok + tt)
    w = F.random_blocks(rng, tt, rows, cols, 0.02)
    q, s = _tokens(rng, n_tok, cols)
    got = rf.gemm_tq_i8(tt, _t(q), _t(s), _t(w), rows, cols).cpu().numpy()
    _check_rows(got, tt, q, s, w, rows, cols)


def test_gemm_all_codes():
    """Random qs bytes: every 2-bit code, 3 included (weight 2)."""
    rng = np.random.default_rng(5)
    rows, cols, n_tok = 190, 1280, 12
    blk = rng.integers(0, 256, size=(rows * cols // 256, 66), dtype=np.uint8)
    d = np.abs(rng.normal(0, 0.02, rows * cols // 256)).astype(np.float16).view(np.uint8)
    blk[:, 64:66] = d.reshape(-1, 2)
    w = blk.reshape(-1)
    q, s = _tokens(rng, n_tok, cols)
    got = rf.gemm_tq_i8(F.TQ2_0, _t(q), _t(s), _t(w), rows, cols).cpu().numpy()
    _check_rows(got, F.TQ2_0, q, s, w, rows, cols)


def test_gemm_packed_equals_gguf_entry():
    rng = np.random.default_rng(9)
    rows, cols, n_tok = 777, 2560, 20
    w = F.random_blocks(rng, F.TQ2_0, rows, cols, 0.02)
    q, s = _tokens(rng, n_tok, cols)
    packed = rf.pack(F.TQ2_0, _t(w), rows, cols)
    a = rf.gemm_tq2_i8_packed(_t(q), _t(s), packed, rows, cols).cpu().numpy()
    b = rf.gemm_tq_i8(F.TQ2_0, _t(q), _t(s), _t(w), rows, cols).cpu().numpy()
    assert np.array_equal(_u32(a), _u32(b))


def test_gemm_equals_device_gemv():
    """The same rows as the single-token device GEMV of the decode path."""
    rng = np.random.default_rng(13)
    rows, cols, n_tok = 2048, 2560, 5
    w = F.random_blocks(rng, F.TQ2_0, rows, cols, 0.02)
    q, s = _tokens(rng, n_tok, cols)
    wd = _t(w)
    got = rf.gemm_tq_i8(F.TQ2_0, _t(q), _t(s), wd, rows, cols).cpu().numpy()
    for t in range(n_tok):
        one = rf.gemv_tq2_i8(_t(q[t]), _t(s[t:t + 1]), wd, rows, cols).cpu().numpy()
        assert np.array_equal(_u32(got[t]), _u32(one))
