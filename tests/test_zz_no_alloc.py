"""foxcuda_gemv_noalloc through the C ABI: the allocation-free variant of
foxcuda_gemv gives the same bits as foxcuda_gemv, on two calls in a row that
share its static scratch, and rejects a matrix larger than that scratch.

The file name sorts last so the test also runs after every other GPU test in
the same process; it passes alone too."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from rustfox_b200 import formats as F  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

DEV = "cuda:0"
SCRATCH_BYTES = 32 << 20  # FOXCUDA_GEMV_NOALLOC_MAX_BYTES in include/foxcuda.h


def _case(tt, rows, cols, seed):
    rng = np.random.default_rng(seed)
    w = torch.from_numpy(F.random_blocks(rng, tt, rows, cols, 0.02)).to(DEV)
    x = torch.from_numpy(rng.normal(0, 1, cols).astype(np.float32)).to(DEV)
    return w, x


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def test_noalloc_matches_gemv_on_two_calls_in_a_row():
    L = rf.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    # call 1 fills 17.4 MB of the scratch; call 2 is smaller, a different
    # type, and a row count that ends in a partial unit, so it runs over the
    # stale bytes call 1 left behind.
    cases = [(F.Q8_0, 32000, 512, 1), (F.TQ1_0, 1000, 2560, 2)]
    inputs = [_case(*c) for c in cases]
    got = [torch.empty(c[1], dtype=torch.float32, device=DEV) for c in cases]
    for (tt, rows, cols, _), (w, x), out in zip(cases, inputs, got):
        assert F.row_bytes(tt, cols) * rows <= SCRATCH_BYTES
        st = L.foxcuda_gemv_noalloc(tt, _ptr(x), _ptr(w), rows, cols, _ptr(out), stream)
        assert st == 0, rf.last_error()
    for (tt, rows, cols, _), (w, x), out in zip(cases, inputs, got):
        want = torch.empty(rows, dtype=torch.float32, device=DEV)
        st = L.foxcuda_gemv(tt, _ptr(x), _ptr(w), rows, cols, _ptr(want), stream)
        assert st == 0, rf.last_error()
        torch.cuda.synchronize()
        a = out.cpu().numpy().view(np.uint32)
        b = want.cpu().numpy().view(np.uint32)
        assert np.array_equal(a, b), f"type {tt}: {np.count_nonzero(a != b)} of {rows} rows differ"


def test_noalloc_rejects_a_matrix_beyond_the_scratch():
    L = rf.lib()
    w, x = _case(F.Q8_0, 64, 2560, 3)
    out = torch.empty(64, dtype=torch.float32, device=DEV)
    rows = 151936  # the 4B head: 413 MB repacked, checked before anything runs
    st = L.foxcuda_gemv_noalloc(F.Q8_0, _ptr(x), _ptr(w), rows, 2560, _ptr(out), None)
    assert st == 1
    assert "static scratch" in rf.last_error()
