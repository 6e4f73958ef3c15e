"""The device's exponential against the host's libm expf, bit for bit.

Upstream's softmax, SwiGLU and sampler call glibc's expf (src/ops.c:24-48,
src/sample.c:162-184). The device restates glibc's published algorithm
(csrc/common.cuh expf_up); here it is evaluated at every float in
[-104, 89] (about 2.24e9 inputs, the range over which expf is neither 0 nor
inf) and at the special values, and compared with libm on the host.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

CHUNK = 1 << 26


def _bits(x: float) -> int:
    return int(np.float32(x).view(np.uint32))


def _sweep(first: int, last: int):
    out = torch.empty(CHUNK, dtype=torch.float32, device="cuda")
    host = torch.empty(CHUNK, dtype=torch.float32, pin_memory=True)
    b = first
    while b <= last:
        n = min(CHUNK, last - b + 1)
        rf.api.expf_range(b, n, out[:n])
        host[:n].copy_(out[:n])
        bad, at = O.expf_mismatches(b, host[:n].numpy())
        assert bad == 0, f"{bad} mismatches from bits {b:#x}, first at {b + at:#x}"
        b += n


def test_every_non_negative_float_up_to_89():
    _sweep(0, _bits(89.0))


def test_every_negative_float_down_to_minus_104():
    _sweep(0x80000000, _bits(-104.0))


def test_special_values():
    xs = np.array([np.inf, -np.inf, np.nan, 0.0, -0.0, 88.7228, 88.72284, 89.5, 1e30, -103.97,
                   -103.98, -150.0, -1e30, 1e-45, -1e-45, 1.17549435e-38], dtype=np.float32)
    for x in xs:
        b = int(x.view(np.uint32))
        got = rf.api.expf_range(b, 1).cpu().numpy()
        bad, _ = O.expf_mismatches(b, got)
        if np.isnan(x):
            assert np.isnan(got[0])
        else:
            assert bad == 0, f"expf({x!r}): device {got[0]!r}"
