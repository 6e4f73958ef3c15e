"""The split form of the tensor-core pass (foxcuda_gemm_tq2_i8_split) against
the oracle and the unsplit pass, bit for bit.

Upstream's forward_batch runs one fox_gemv_tq{1,2}_i8 per token
(src/forward.c:188-213); the split pass must give each token that GEMV's row.
The cases cover one and several blocks per CTA, ragged rows and tokens, and
the 4B layer shapes at verification sizes.
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


CASES = [(200, 768, 9), (130, 512, 3), (2560, 9728, 8), (19456, 2560, 8), (6144, 2560, 16),
         (300, 2560, 1), (1000, 21504, 5)]


@pytest.mark.parametrize("rows,cols,n_tok", CASES)
def test_split_equals_oracle_and_unsplit(rows, cols, n_tok):
    rng = np.random.default_rng(rows + cols + n_tok)
    w = F.random_blocks(rng, F.TQ2_0, rows, cols, 0.02)
    q = np.empty((n_tok, cols), dtype=np.int8)
    s = np.empty(n_tok, dtype=np.float32)
    for t in range(n_tok):
        q[t], s[t] = O.quantize_i8(rng.normal(0, 1, cols).astype(np.float32))
    packed = rf.pack(F.TQ2_0, _t(w), rows, cols)
    split = rf.gemm_tq2_i8_split(_t(q), _t(s), packed, rows, cols).cpu().numpy()
    whole = rf.gemm_tq2_i8_packed(_t(q), _t(s), packed, rows, cols).cpu().numpy()
    assert np.array_equal(_u32(split), _u32(whole))
    for t in range(min(n_tok, 3)):
        want = O.gemv_tq_i8(F.TQ2_0, q[t], float(s[t]), w, rows, cols)
        assert np.array_equal(_u32(split[t]), _u32(want))
