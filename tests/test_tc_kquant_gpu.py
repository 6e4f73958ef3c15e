"""The K-quant tensor-core pass (foxcuda_gemm_kq_i8, tcgen05 kind::i8 on
Q4_K and Q6_K) against the oracle, bit for bit.

Upstream's forward_batch runs one K-quant GEMV per token (src/forward.c:
188-213, src/kernels.c:571-805), each token quantised with one scale per 256
block (src/kernels.c:722-754). The pass must give each token that GEMV's row.
The cases cover both types, one and several token tiles, ragged rows, and
config 3's shapes at the M = 8 of its verification pass.
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


CASES = [
    (F.Q4_K, 37, 512, 3), (F.Q4_K, 200, 1024, 12), (F.Q4_K, 4096, 4096, 8),
    (F.Q4_K, 4096, 14336, 8), (F.Q4_K, 300, 4096, 33),
    (F.Q6_K, 37, 512, 3), (F.Q6_K, 1024, 4096, 8), (F.Q6_K, 130, 2048, 20),
]


@pytest.mark.parametrize("tt,rows,cols,n_tok", CASES)
def test_kquant_pass_equals_per_token_gemv(tt, rows, cols, n_tok):
    rng = np.random.default_rng(rows + cols + n_tok + tt)
    w = F.random_blocks(rng, tt, rows, cols, 0.01)
    xs = [rng.normal(0, 1, cols).astype(np.float32) for _ in range(n_tok)]
    q = np.empty((n_tok, cols), dtype=np.int8)
    s = np.empty((n_tok, cols // 256), dtype=np.float32)
    for t, x in enumerate(xs):
        q[t], s[t] = O.quantize_k(x)
    got = rf.gemm_kq_i8(tt, _t(q), _t(s), _t(w), rows, cols).cpu().numpy()
    for t, x in enumerate(xs):
        want = O.gemv(tt, x, w, rows, cols)
        bad = np.count_nonzero(_u32(got[t]) != _u32(want))
        assert bad == 0, f"token {t}: {bad} of {rows} rows differ; max |d| {np.abs(got[t] - want).max()}"
