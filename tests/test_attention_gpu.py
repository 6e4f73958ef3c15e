"""Decode attention through the C ABI (foxcuda_attention).

Upstream's attention_heads (src/forward.c:222-257 in the RustFox tree): per
query head, scores q.k_j * (1/sqrtf(hd)) for j <= pos, fox_softmax
(src/ops.c:24-39), then out = sum_j a_j v_j, each sum serial in float.

  exact = 1  must equal that serial order bit for bit. The reference here is
             numpy float32 in the same order, with the oracle's softmax
             (libm's expf, which the device's exponential reproduces).
  exact = 0  is the tile attention of the decode step. It sums in another
             order, which the oracle restates (oracle.tile_attention): bit
             for bit against that, and within 1e-5 of the output's scale
             against a float64 torch reference.
Both run on fp32 and fp16 caches (fp16 values are exactly representable in
fp32, so the references read the same numbers).
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from oracle import oracle as O  # noqa: E402
import rustfox_b200 as rf  # noqa: E402

DEV = "cuda:0"
CASES = [  # n_head, n_kv, head_dim, n_ctx, pos
    (8, 2, 64, 64, 0), (8, 2, 64, 256, 37), (8, 2, 64, 256, 255),
    (32, 8, 128, 1024, 31), (32, 8, 128, 1024, 511), (32, 8, 128, 4096, 4095),
    (32, 4, 128, 512, 300), (16, 2, 128, 256, 200),
]


def _inputs(n_head, n_kv, hd, n_ctx, seed, f16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(n_head * hd, generator=g)
    k = torch.randn(n_kv, n_ctx, hd, generator=g)
    v = torch.randn(n_kv, n_ctx, hd, generator=g)
    if f16:
        k, v = k.half(), v.half()
    return q, k, v


def _run(q, k, v, n_head, n_kv, hd, n_ctx, pos, exact, f16):
    out = torch.full((n_head * hd,), float("nan"), device=DEV)
    qd, kd, vd = q.to(DEV), k.to(DEV).contiguous(), v.to(DEV).contiguous()
    st = rf.lib().foxcuda_attention(C.c_void_p(qd.data_ptr()), C.c_void_p(kd.data_ptr()),
                                    C.c_void_p(vd.data_ptr()), 0 if f16 else 1, n_head, n_kv, hd,
                                    n_ctx, pos, exact, C.c_void_p(out.data_ptr()), None)
    assert st == 0, rf.last_error()
    torch.cuda.synchronize()
    return out.cpu()


def _ref64(q, k, v, n_head, n_kv, hd, pos):
    gqa = n_head // n_kv
    qh = q.double().view(n_head, hd)
    kk = k.double()[:, : pos + 1].repeat_interleave(gqa, 0)
    vv = v.double()[:, : pos + 1].repeat_interleave(gqa, 0)
    s = torch.einsum("hd,hjd->hj", qh, kk) * (1.0 / np.sqrt(hd))
    a = torch.softmax(s, dim=-1)
    return torch.einsum("hj,hjd->hd", a, vv).reshape(-1)


def _ref_serial(q, k, v, n_head, n_kv, hd, pos):
    """upstream's order in float32 (no fused multiply-add)."""
    L = O.lib()
    L.or_softmax.argtypes = [C.c_void_p, C.c_size_t]
    gqa = n_head // n_kv
    qn = q.numpy().astype(np.float32).reshape(n_head, hd)
    kn = k.float().numpy()
    vn = v.float().numpy()
    scale = np.float32(1.0) / np.sqrt(np.float32(hd), dtype=np.float32)
    out = np.zeros((n_head, hd), np.float32)
    for h in range(n_head):
        K = kn[h // gqa, : pos + 1]
        V = vn[h // gqa, : pos + 1]
        s = np.zeros(pos + 1, np.float32)
        for d in range(hd):  # s_j += q[d] * k_j[d], j vectorised, each step rounded
            s = (s + (qn[h, d] * K[:, d]).astype(np.float32)).astype(np.float32)
        att = np.ascontiguousarray((s * scale).astype(np.float32))
        L.or_softmax(att.ctypes.data_as(C.c_void_p), att.size)
        acc = np.zeros(hd, np.float32)
        for j in range(pos + 1):
            acc = (acc + (att[j] * V[j]).astype(np.float32)).astype(np.float32)
        out[h] = acc
    return out.reshape(-1)


@pytest.mark.parametrize("f16", [True, False])
@pytest.mark.parametrize("case", CASES)
def test_tile_kernel_matches_fp64(case, f16):
    n_head, n_kv, hd, n_ctx, pos = case
    q, k, v = _inputs(n_head, n_kv, hd, n_ctx, pos + hd, f16)
    got = _run(q, k, v, n_head, n_kv, hd, n_ctx, pos, 0, f16).double()
    want = _ref64(q, k, v, n_head, n_kv, hd, pos)
    err = (got - want).abs().max().item() / want.abs().max().item()
    assert err <= 1e-5, err


@pytest.mark.parametrize("f16", [True, False])
@pytest.mark.parametrize("case", CASES)
def test_tile_kernel_is_the_oracles_tile_order(case, f16):
    n_head, n_kv, hd, n_ctx, pos = case
    q, k, v = _inputs(n_head, n_kv, hd, n_ctx, pos + 3 * hd, f16)
    got = _run(q, k, v, n_head, n_kv, hd, n_ctx, pos, 0, f16).numpy()
    nt = rf.lib().foxcuda_attn_tile_target(0, n_kv)
    gqa = n_head // n_kv
    qn = q.numpy().astype(np.float32).reshape(n_head, hd)
    kn, vn = k.float().numpy(), v.float().numpy()
    scale = np.float32(1.0) / np.sqrt(np.float32(hd), dtype=np.float32)
    want = np.concatenate([O.tile_attention(qn[h], kn[h // gqa, : pos + 1], vn[h // gqa, : pos + 1], nt,
                                            float(scale)) for h in range(n_head)])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (
        f"{np.count_nonzero(got != want)} of {got.size} differ")


@pytest.mark.parametrize("f16", [True, False])
@pytest.mark.parametrize("case", [c for c in CASES if c[4] <= 600])
def test_exact_kernel_is_upstream_order(case, f16):
    n_head, n_kv, hd, n_ctx, pos = case
    q, k, v = _inputs(n_head, n_kv, hd, n_ctx, pos + 7, f16)
    got = _run(q, k, v, n_head, n_kv, hd, n_ctx, pos, 1, f16).numpy()
    want = _ref_serial(q, k, v, n_head, n_kv, hd, pos)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (
        f"{np.count_nonzero(got != want)} of {got.size} differ")


def test_rejects_bad_shapes():
    q = torch.zeros(8 * 64, device=DEV)
    k = torch.zeros(2, 16, 64, device=DEV)
    L = rf.lib()
    p = C.c_void_p
    assert L.foxcuda_attention(p(q.data_ptr()), p(k.data_ptr()), p(k.data_ptr()), 1, 8, 3, 64, 16,
                               0, 0, p(q.data_ptr()), None) == 5  # 8 heads over 3 kv heads
    assert L.foxcuda_attention(p(q.data_ptr()), p(k.data_ptr()), p(k.data_ptr()), 1, 8, 2, 64, 16,
                               16, 0, p(q.data_ptr()), None) == 1  # position beyond the cache
