"""GPU parity of the kernel tier against the oracle: bit-exact int32 for
igemm s8s8/u8s8 and bit-exact f32 for the int4 packed GEMM (integer group
dots, then the same sequential f32 sum).  All calls go through the C ABI."""
import numpy as np
import pytest

from tests.refrng import Xs64, pseudo_i8, pseudo_u8

pytestmark = pytest.mark.gpu


def i64_ref(a, b, m, k, n):
    return (a.reshape(m, k).astype(np.int64) @ b.reshape(n, k).astype(np.int64).T).reshape(-1)


def test_selftest_battery(cuda):
    from franken_ocr_b200 import simd

    rep = simd.selftest()
    assert rep["cases_total"] == 24
    bad = [c for c in rep["cases"] if not c["ok"]]
    assert rep["all_ok"] and not bad, bad


def test_hand_values_and_accumulate(cuda):
    from franken_ocr_b200 import simd

    out = np.zeros(4, np.int32)
    simd.igemm_s8s8(np.array([1, 2, 3, 4, 5, 6], np.int8), np.array([1, 0, 1, 0, 1, 0], np.int8),
                    2, 3, 2, out)
    assert out.tolist() == [4, 2, 10, 5]
    out = np.array([100], np.int32)
    simd.igemm_s8s8(np.array([1, 2, 3], np.int8), np.array([1, 1, 1], np.int8), 1, 3, 1, out)
    simd.igemm_s8s8(np.array([1, 2, 3], np.int8), np.array([1, 1, 1], np.int8), 1, 3, 1, out)
    assert out.tolist() == [112]
    out = np.zeros(1, np.int32)
    simd.igemm_u8s8(np.array([10, 20, 30], np.uint8), np.array([2, -1, 1], np.int8), 1, 3, 1, out)
    assert out.tolist() == [30]


@pytest.mark.parametrize("u8", [False, True])
def test_batched_sweep(cuda, oracle, u8):
    """tests/batched_igemm_parity.rs M/N/K sweep (+= onto a seeded out)."""
    from franken_ocr_b200 import simd

    rng = Xs64(0xC0FFEE1234 + u8)
    Ms = [1, 2, 3, 4, 5, 6, 7, 8, 9, 15, 16, 17, 31, 32, 33, 63, 64, 65, 127, 128, 129, 256]
    for m in Ms:
        for n in (1, 4, 5, 7, 10, 64, 65):
            for k in (1, 16, 17, 128):
                a = rng.fill_i8(m * k)
                if u8:
                    a = a.view(np.uint8)
                b = rng.fill_i8(n * k)
                seed = np.arange(m * n, dtype=np.int32) - 7
                got = seed.copy()
                (simd.igemm_u8s8 if u8 else simd.igemm_s8s8)(a, b, m, k, n, got)
                want = seed.copy()
                (oracle.igemm_u8s8 if u8 else oracle.igemm_s8s8)(a, b, m, k, n, want)
                assert np.array_equal(got, want), (m, n, k)


def test_decode_shapes_and_k6848(cuda, oracle):
    """tests/batched_decode_bit_identity.rs shapes + the K=6848 worst case."""
    from franken_ocr_b200 import simd

    for (n, k) in [(3840, 1280), (1280, 1280), (896, 1280), (1280, 896), (1280, 6848), (512, 1280)]:
        for m in (1, 4, 8, 9):
            a, b = pseudo_i8(m * k, n + m), pseudo_i8(n * k, k + m)
            got = np.zeros(m * n, np.int32)
            simd.igemm_s8s8(a, b, m, k, n, got)
            assert np.array_equal(got.astype(np.int64), i64_ref(a, b, m, k, n)), (m, n, k)
    k = 6848
    got = np.zeros(4, np.int32)
    simd.igemm_u8s8(np.full(k, 255, np.uint8), np.full(4 * k, -128, np.int8), 1, k, 4, got)
    assert (got == -223_518_720).all()


@pytest.mark.parametrize("n,k", [(1792, 1280), (1280, 896), (129280, 1280)])
@pytest.mark.parametrize("m", [1, 4, 8, 64, 512, 4096])
def test_config1_sweep_device(cuda, m, n, k):
    """Config 1 (raw GEMM sweep) on device tensors; exact on sampled rows and
    on the size-independent checksum sum_n out[m,n] == a[m] . sum_n b[n]."""
    import torch

    from franken_ocr_b200 import simd

    g = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    a = torch.randint(-127, 128, (m, k), dtype=torch.int8, device="cuda", generator=g)
    b = torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda", generator=g)
    out = torch.zeros((m, n), dtype=torch.int32, device="cuda")
    simd.igemm_s8s8(a, b, m, k, n, out)
    torch.cuda.synchronize()
    a64, b64 = a.to(torch.int64).cpu(), b.to(torch.int64).cpu()
    chk = a64 @ b.to(torch.int64).sum(0).cpu()
    assert torch.equal(out.to(torch.int64).sum(1).cpu(), chk)
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(1))[:4]
    cols = torch.randperm(n, generator=torch.Generator().manual_seed(2))[:512]
    ref = a64[rows] @ b64[cols].T
    assert torch.equal(out[rows][:, cols].cpu().to(torch.int64), ref)


@pytest.mark.parametrize("m,n,k", [(512, 1280, 896), (4096, 1792, 1280), (48, 1792, 1280)])
def test_u8s8_tensor_cores(cuda, m, n, k):
    """igemm_u8s8 (dispatch.rs:276) at tensor-core shapes: unsigned activations
    in [0, 255] (the MMA's A operand unsigned, B signed), += onto a seeded out,
    every element exact against an int64 product."""
    import torch

    from franken_ocr_b200 import simd

    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randint(0, 256, (m, k), dtype=torch.uint8, device="cuda", generator=g)
    b = torch.randint(-128, 128, (n, k), dtype=torch.int8, device="cuda", generator=g)
    seed = torch.arange(m * n, dtype=torch.int32, device="cuda").reshape(m, n) - 1000
    out = seed.clone()
    simd.igemm_u8s8(a, b, m, k, n, out)
    torch.cuda.synchronize()
    ref = a.cpu().to(torch.int64) @ b.cpu().to(torch.int64).T + seed.cpu().to(torch.int64)
    assert torch.equal(out.cpu().to(torch.int64), ref)


def test_int4_cases(cuda, oracle):
    """tests/int4_packed_parity.rs cases, K=6848 worst case and the config-4
    shapes: bit-identical f32 to the oracle; out is overwritten."""
    from franken_ocr_b200 import simd

    rng = Xs64(0x1A2B3C4D5E6F7081)
    cases = [(1, 16, 1, 16), (1, 32, 1, 32), (2, 32, 3, 16), (3, 48, 2, 16), (4, 64, 5, 32),
             (5, 96, 7, 16), (7, 128, 6, 32), (8, 160, 9, 16), (9, 16, 4, 16), (16, 64, 13, 16),
             (17, 32, 5, 32), (33, 48, 3, 16), (4, 6848, 5, 16), (9, 6848, 3, 32),
             (1, 1280, 896, 32), (1, 896, 1280, 32), (8, 1280, 1792, 32)]
    for m, k, n, group in cases:
        a = rng.fill_i8q(m * k)
        bp = np.random.default_rng(m * k + n).integers(0, 256, n * (k // 2), dtype=np.uint8)
        sc = rng.fill_scales(n * (k // group))
        got = np.full(m * n, 123.5, np.float32)
        simd.igemm_s4s8_packed(a, bp, sc, group, m, k, n, got)
        want = oracle.igemm_s4s8_packed(a, bp, sc, group, m, k, n)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (m, k, n, group)


def test_quantize_rows_and_gemv(cuda, oracle):
    from franken_ocr_b200 import simd

    g = np.random.default_rng(3)
    x = g.standard_normal((5, 1280), dtype=np.float32)
    x[1] = 0.0
    x[2, :8] = [-127.0, -2.5, -1.5, -0.5, 0.5, 1.5, 2.5, 127.0]
    x[2, 8:] = 0.0
    for te in (False, True):
        xq = np.empty_like(x, dtype=np.int8)
        sc = np.empty(5, np.float32)
        simd.quantize_rows_i8(x, 5, 1280, xq, sc, ties_even=te)
        for r in range(5):
            q, s = oracle.quantize_row_i8(x[r], ties_even=te)
            assert np.array_equal(xq[r], q) and sc[r] == s
    w = g.integers(-127, 128, (896, 1280), dtype=np.int8)
    ws = g.uniform(0.001, 0.02, 896).astype(np.float32)
    y = np.empty((5, 896), np.float32)
    simd.gemv_i8(x, 5, 1280, w, ws, 896, y)
    for r in range(5):
        assert np.array_equal(y[r].view(np.uint32), oracle.gemv_i8(x[r], w, ws).view(np.uint32))


@pytest.mark.parametrize("m,n,k", [(300, 1000, 256), (129, 130, 144), (257, 260, 128),
                                   (4096, 1792, 1280), (640, 6000, 896),
                                   (64, 1792, 1280), (9, 700, 96), (100, 40000, 1024),
                                   (37, 33000, 1040)])
def test_tc_accumulate_ragged(cuda, m, n, k):
    """+= onto a seeded int32 out with ragged edges on every multi-row route:
    the tensor-core path with the TMA reduce-add epilogue (N % 4 == 0) and
    the per-row one (N % 4 != 0); 8 < M < 128 through the chunked GEMV grid
    (small weights) and through the tensor-core path, whose 128-row A boxes
    run past row M and read zeros there (weights of 32 MB and more, and any
    M > 16)."""
    import torch

    from franken_ocr_b200 import simd

    g = torch.Generator(device="cuda").manual_seed(m + 31 * n + k)
    a = torch.randint(-127, 128, (m, k), dtype=torch.int8, device="cuda", generator=g)
    b = torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda", generator=g)
    seed = torch.randint(-1000, 1000, (m, n), dtype=torch.int32, device="cuda", generator=g)
    out = seed.clone()
    simd.igemm_s8s8(a, b, m, k, n, out)
    torch.cuda.synchronize()
    a64, b64, s64 = a.to(torch.int64).cpu(), b.to(torch.int64).cpu(), seed.to(torch.int64).cpu()
    o64 = out.to(torch.int64).cpu()
    if m * n * k <= 1 << 28:
        assert torch.equal(o64, a64 @ b64.T + s64)
    else:
        assert torch.equal(o64.sum(1), a64 @ b64.sum(0) + s64.sum(1))
        rows = torch.cat([torch.arange(4), torch.arange(m - 4, m)])
        assert torch.equal(o64[rows], a64[rows] @ b64.T + s64[rows])


@pytest.mark.parametrize("m,k,n,group", [
    (64, 1280, 1792, 32), (256, 1280, 896, 32), (256, 896, 1280, 32), (65, 1280, 16160, 32),
    (32, 1280, 1792, 16), (100, 896, 1280, 16), (256, 1280, 130, 16), (300, 128, 257, 32)])
def test_int4_tensor_core_shapes(cuda, oracle, m, k, n, group):
    """The tcgen05 int4 path (M >= 64, or 32 for groups of 16; K a multiple of
    128): bit-identical to the oracle in host and device mode, ragged M and N
    included."""
    import torch

    from franken_ocr_b200 import simd

    g = np.random.default_rng(m * 7 + n)
    a = g.integers(-127, 128, m * k, dtype=np.int8)
    bp = g.integers(0, 256, n * (k // 2), dtype=np.uint8)
    sc = g.uniform(0.001, 0.02, n * (k // group)).astype(np.float32)
    want = oracle.igemm_s4s8_packed(a, bp, sc, group, m, k, n)
    got = np.full(m * n, 123.5, np.float32)
    simd.igemm_s4s8_packed(a, bp, sc, group, m, k, n, got)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    da, db, ds = (torch.from_numpy(v).cuda() for v in (a, bp, sc))
    dout = torch.full((m * n,), float("nan"), device="cuda")
    simd.igemm_s4s8_packed(da, db, ds, group, m, k, n, dout)
    torch.cuda.synchronize()
    assert np.array_equal(dout.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_int4_tensor_core_extremes(cuda, oracle):
    """All weights -8 against +-127 activations: every group dot at its
    extreme (-32512 / +32512 for groups of 32), through the tcgen05 path."""
    from franken_ocr_b200 import simd

    m, k, n = 64, 1280, 256
    for group in (16, 32):
        a = np.where(np.arange(m * k) % 3 == 0, -127, 127).astype(np.int8)
        bp = np.full(n * (k // 2), 0x88, np.uint8)
        sc = np.linspace(0.001, 0.05, n * (k // group)).astype(np.float32)
        got = np.empty(m * n, np.float32)
        simd.igemm_s4s8_packed(a, bp, sc, group, m, k, n, got)
        want = oracle.igemm_s4s8_packed(a, bp, sc, group, m, k, n)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), group


def test_igemm_status_query_clean(cuda):
    """After tensor-core igemm calls the device status word is 0."""
    import ctypes as C

    import torch

    from franken_ocr_b200 import simd
    from franken_ocr_b200._lib import check, lib

    a = torch.randint(-127, 128, (256, 1280), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (1792, 1280), dtype=torch.int8, device="cuda")
    o = torch.zeros((256, 1792), dtype=torch.int32, device="cuda")
    simd.igemm_s8s8(a, b, 256, 1280, 1792, o)
    torch.cuda.synchronize()
    w = C.c_int(-1)
    check(lib.focr_igemm_status(C.byref(w), 1))
    assert w.value == 0
