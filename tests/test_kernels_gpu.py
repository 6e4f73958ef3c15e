"""Kernel-level parity of libfoxcuda against the CPU oracle (bit-exact).

Mirrors upstream's own kernel tests (tests/test_ternary.c, test_gemv.c,
test_kernels.c in the RustFox tree) on the device: known answers, exact
element order, serial == parallel, the float entry == the pre-quantised entry,
argument rejection. Every GEMV here is compared bit for bit: the integer block
sums are order-free and the float terms are accumulated in upstream's order.
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


SHAPES = [
    (F.TQ1_0, 37, 512), (F.TQ1_0, 6144, 2560), (F.TQ1_0, 2560, 9728), (F.TQ1_0, 64, 256),
    (F.TQ2_0, 37, 512), (F.TQ2_0, 1024, 5120), (F.TQ2_0, 512, 21504),
    (F.Q4_K, 37, 512), (F.Q4_K, 1024, 4096), (F.Q4_K, 256, 14336),
    (F.Q6_K, 37, 512), (F.Q6_K, 1024, 4096),
    (F.Q8_0, 37, 512), (F.Q8_0, 2048, 2560), (F.Q8_0, 256, 5120),
]


@pytest.mark.parametrize("tt,rows,cols", SHAPES)
def test_gemv_bit_exact(tt, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols + tt)
    w = F.random_blocks(rng, tt, rows, cols, 0.02)
    x = rng.normal(0, 1, cols).astype(np.float32)
    want = O.gemv(tt, x, w, rows, cols)
    got = rf.gemv(tt, _t(x), _t(w), rows, cols).cpu().numpy()
    torch.cuda.synchronize()
    assert np.array_equal(_u32(got), _u32(want)), (
        f"{np.count_nonzero(_u32(got) != _u32(want))} of {rows} rows differ; "
        f"max |d| {np.abs(got - want).max()}")


@pytest.mark.parametrize("tt,rows,cols", [s for s in SHAPES if s[0] != F.Q8_0])
def test_block_partials_bit_exact(tt, rows, cols):
    rng = np.random.default_rng(rows + cols * 3 + tt)
    w = F.random_blocks(rng, tt, rows, cols, 0.02)
    q = rng.integers(-127, 128, size=cols, dtype=np.int8)
    want = O.block_partials(tt, q, w, rows, cols)
    got = rf.block_partials(tt, _t(q), _t(w), rows, cols).cpu().numpy()
    assert np.array_equal(got, want)


@pytest.mark.parametrize("tt,rows,cols", [(F.TQ1_0, 37, 512), (F.TQ1_0, 4096, 2560),
                                          (F.TQ2_0, 37, 512), (F.TQ2_0, 5120, 4096)])
def test_gemv_i8_entry(tt, rows, cols):
    """fox_gemv_tq{1,2}_i8 with pre-quantised activations; also equal to the
    float entry point (upstream test_gemv.c:145-152)."""
    rng = np.random.default_rng(11 + rows)
    w = F.random_blocks(rng, tt, rows, cols, 0.02)
    x = (rng.integers(0, 256, size=cols) - 128).astype(np.float32) * 0.01
    q, s = O.quantize_i8(x)
    want = O.gemv_tq_i8(tt, q, s, w, rows, cols)
    fn = rf.gemv_tq1_i8 if tt == F.TQ1_0 else rf.gemv_tq2_i8
    got = fn(_t(q), _t(np.array([s], dtype=np.float32)), _t(w), rows, cols).cpu().numpy()
    assert np.array_equal(_u32(got), _u32(want))
    flt = rf.gemv(tt, _t(x), _t(w), rows, cols).cpu().numpy()
    assert np.array_equal(_u32(flt), _u32(want))


def test_packed_entry_equals_gguf_entry():
    rng = np.random.default_rng(3)
    for tt, rows, cols in [(F.TQ1_0, 96, 2560), (F.Q4_K, 64, 4096), (F.Q8_0, 80, 2560)]:
        w = F.random_blocks(rng, tt, rows, cols, 0.02)
        x = _t(rng.normal(0, 1, cols).astype(np.float32))
        wt = _t(w)
        packed = rf.pack(tt, wt, rows, cols)
        assert packed.numel() == w.size
        a = rf.gemv(tt, x, wt, rows, cols).cpu().numpy()
        b = rf.gemv_packed(tt, x, packed, rows, cols).cpu().numpy()
        assert np.array_equal(_u32(a), _u32(b))
        assert sorted(packed.cpu().numpy().tolist()) == sorted(w.tolist())  # a permutation


@pytest.mark.parametrize("n", [256, 2560, 9728, 37])
def test_quantize_bit_exact(n):
    rng = np.random.default_rng(n)
    x = rng.normal(0, 3, n).astype(np.float32)
    x[n // 2] = 0.0
    q, s = rf.quantize_activations_i8(_t(x))
    wq, ws = O.quantize_i8(x)
    assert np.array_equal(q.cpu().numpy(), wq)
    assert _u32(s.cpu().numpy()[0]) == _u32(ws)


def test_quantize_edge_cases():
    """upstream test_gemv.c:81-94: zero vector -> zero scale; the largest
    magnitude maps to 127; every value inside the int8 range."""
    z = _t(np.zeros(512, np.float32))
    q, s = rf.quantize_activations_i8(z)
    assert float(s.cpu()[0]) == 0.0 and not q.cpu().numpy().any()
    x = np.arange(512, dtype=np.float32) - 200.0
    q, s = rf.quantize_activations_i8(_t(x))
    qn = q.cpu().numpy()
    assert qn[-1] == 127 and qn.min() >= -127 and float(s.cpu()[0]) > 0


@pytest.mark.parametrize("tt,n", [(F.Q8_0, 2560), (F.Q4_K, 512), (F.Q6_K, 512), (F.F16, 64),
                                  (F.F32, 64)])
def test_dequant_row_bit_exact(tt, n):
    rng = np.random.default_rng(n + tt)
    if tt == F.F32:
        row = rng.normal(0, 1, n).astype(np.float32)
    elif tt == F.F16:
        row = rng.normal(0, 1, n).astype(np.float16)
    else:
        row = F.random_blocks(rng, tt, 1, n, 0.02)
    want = O.dequant_row(tt, row, n)
    got = rf.dequant_row(tt, _t(row.view(np.uint8)), n).cpu().numpy()
    assert np.array_equal(_u32(got), _u32(want))


def test_tq_known_answers():
    """upstream test_ternary.c:95-136: an all-plus-one block against all-ones
    activations sums to N, an all-zero block to -N."""
    nblk = 3
    n = 256 * nblk
    ones = _t(np.ones(n, np.int8))
    one_scale = _t(np.array([1.0], np.float32))
    tq1 = np.zeros((nblk, 54), np.uint8)
    tq1[:, :48] = 255
    tq1[:, 48:52] = 253
    tq1[:, 52:54] = [0x00, 0x3C]
    tq2 = np.zeros((nblk, 66), np.uint8)
    tq2[:, :64] = 0xAA
    tq2[:, 64:66] = [0x00, 0x3C]
    assert float(rf.gemv_tq1_i8(ones, one_scale, _t(tq1.reshape(-1)), 1, n).cpu()[0]) == n
    assert float(rf.gemv_tq2_i8(ones, one_scale, _t(tq2.reshape(-1)), 1, n).cpu()[0]) == n
    tq1[:, :52] = 0
    tq2[:, :64] = 0
    assert float(rf.gemv_tq1_i8(ones, one_scale, _t(tq1.reshape(-1)), 1, n).cpu()[0]) == -n
    assert float(rf.gemv_tq2_i8(ones, one_scale, _t(tq2.reshape(-1)), 1, n).cpu()[0]) == -n


def test_argument_rejection():
    """upstream test_gemv.c:309-316 / test_kernels.c:369-374: ragged columns,
    null pointers and unsupported types are refused with a status."""
    x = _t(np.ones(512, np.float32))
    w = _t(np.zeros(37 * 2 * 66, np.uint8))
    with pytest.raises(rf.FoxError) as e:
        rf.gemv(F.TQ2_0, x, w, 37, 255)
    assert e.value.status == 1
    assert rf.lib().foxcuda_gemv(F.TQ2_0, None, rf.api._dp(w), 37, 512, rf.api._dp(x),
                                 None) == 1  # null activations
    with pytest.raises(rf.FoxError) as e:
        rf.gemv(10, x, w, 1, 256)  # Q2_K
    assert e.value.status == 5
    with pytest.raises(rf.FoxError) as e:
        rf.gemv(F.TQ1_0, x, w, 0, 512)
    assert e.value.status == 1
    with pytest.raises(rf.FoxError) as e:
        rf.dequant_row(F.TQ1_0, w, 256)
    assert e.value.status == 5
