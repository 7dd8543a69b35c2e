"""Pin the CPU oracle to the reference's own known-answer tests.

Each test restates a reference test (cited) and checks the oracle against the
hand-computed values it asserts.  The reference (Rust) cannot be built here,
so these KATs are what pins the oracle.
"""
import math

import numpy as np
import pytest

from tests.refrng import Xs64, pseudo_i8, pseudo_u8, rotl32, xs32_stream


def i64_ref(a, b, m, k, n):
    return (a.reshape(m, k).astype(np.int64) @ b.reshape(n, k).astype(np.int64).T).reshape(-1)


# ---- src/simd/scalar.rs tests --------------------------------------------

def test_s8s8_hand_computed(oracle):
    out = np.zeros(4, np.int32)
    oracle.igemm_s8s8(np.array([1, 2, 3, 4, 5, 6], np.int8), np.array([1, 0, 1, 0, 1, 0], np.int8),
                      2, 3, 2, out)
    assert out.tolist() == [4, 2, 10, 5]


def test_s8s8_accumulates(oracle):
    out = np.array([100], np.int32)
    a, b = np.array([1, 2, 3], np.int8), np.array([1, 1, 1], np.int8)
    oracle.igemm_s8s8(a, b, 1, 3, 1, out)
    assert out.tolist() == [106]
    oracle.igemm_s8s8(a, b, 1, 3, 1, out)
    assert out.tolist() == [112]


def test_u8s8_hand_and_negatives(oracle):
    out = np.zeros(1, np.int32)
    oracle.igemm_u8s8(np.array([10, 20, 30], np.uint8), np.array([2, -1, 1], np.int8), 1, 3, 1, out)
    assert out.tolist() == [30]
    out = np.zeros(2, np.int32)
    oracle.igemm_s8s8(np.array([-2, 3], np.int8), np.array([-1, -1, 4, -2], np.int8), 1, 2, 2, out)
    assert out.tolist() == [-1, -14]


@pytest.mark.parametrize("av,bv,u8,want", [
    (127, 127, False, 110_451_392), (-128, -128, False, 112_197_632),
    (255, 127, True, 221_772_480), (255, -128, True, -223_518_720)])
def test_k6848_extremes(oracle, av, bv, u8, want):
    K = 6848
    out = np.zeros(4 if bv == -128 and u8 else 1, np.int32)
    n = out.size
    a = np.full(K, av, np.uint8 if u8 else np.int8)
    b = np.full(n * K, bv, np.int8)
    (oracle.igemm_u8s8 if u8 else oracle.igemm_s8s8)(a, b, 1, K, n, out)
    assert (out == want).all()


def test_randomized_vs_i64(oracle):
    m, k, n = 3, 17, 5
    a, b = pseudo_i8(m * k, 0x12345678), pseudo_i8(n * k, 0x9ABCDEF0)
    out = np.zeros(m * n, np.int32)
    oracle.igemm_s8s8(a, b, m, k, n, out)
    assert (out.astype(np.int64) == i64_ref(a, b, m, k, n)).all()
    m, k, n = 4, 13, 6
    a, b = pseudo_u8(m * k, 0x0F0F1234), pseudo_i8(n * k, 0xFEEDFACE)
    out = np.zeros(m * n, np.int32)
    oracle.igemm_u8s8(a, b, m, k, n, out)
    assert (out.astype(np.int64) == i64_ref(a, b, m, k, n)).all()


def test_cpu_baseline_bit_identical(oracle):
    """The timed baseline (restated AVX-512-VNNI tier) equals the oracle,
    including K tails that straddle the 64-byte chunk (x86.rs:983-1142)."""
    for (m, k, n, seed) in [(1, 63, 3, 1), (2, 64, 5, 2), (3, 65, 4, 3), (5, 1280, 7, 4),
                            (1, 6848, 4, 5), (4, 33, 5, 6)]:
        a, b = pseudo_i8(m * k, seed), pseudo_i8(n * k, seed + 99)
        want = np.zeros(m * n, np.int32)
        got = np.zeros(m * n, np.int32)
        oracle.igemm_s8s8(a, b, m, k, n, want)
        oracle.cpu_igemm_s8s8(a, b, m, k, n, got)
        assert (got == want).all()


# ---- dispatch.rs selftest battery: xorshift32 fills reproduce ------------

def test_selftest_seed_streams():
    # u8 domain uses seed.rotate_left(7) | 1 (dispatch.rs:395-404)
    assert rotl32(0x11111111, 7) == 0x88888888
    v, _ = xs32_stream(0x11111111 | 1, 2)
    assert v.dtype == np.uint32 and v[0] != v[1]


# ---- src/simd/int4.rs tests + tests/int4_packed_parity.rs ----------------

def test_nibble_sign_extension(oracle):
    expected = [0, 1, 2, 3, 4, 5, 6, 7, -8, -7, -6, -5, -4, -3, -2, -1]
    assert [oracle.sign_extend_nibble(n) for n in range(16)] == expected


@pytest.mark.parametrize("byte,lo,hi", [(0x21, 1, 2), (0x43, 3, 4), (0x87, 7, -8), (0xF0, 0, -1),
                                        (0x00, 0, 0), (0x88, -8, -8)])
def test_unpack_byte(oracle, byte, lo, hi):
    assert oracle.unpack_to_i8([byte], 1, 2).tolist() == [lo, hi]


def test_unpack_fixtures(oracle):
    assert oracle.unpack_to_i8([0x21, 0x43], 1, 4).tolist() == [1, 2, 3, 4]
    assert oracle.unpack_to_i8([0x21, 0x43, 0x65, 0x87], 2, 4).tolist() == [1, 2, 3, 4, 5, 6, 7, -8]


def spec_packed(a, bp, scales, group, m, k, n):
    """Independent spec oracle (tests/int4_packed_parity.rs oracle_packed_f32)."""
    q = np.empty((n, k), np.int64)
    lo = (bp.reshape(n, k // 2) & 0xF).astype(np.int64)
    hi = (bp.reshape(n, k // 2) >> 4).astype(np.int64)
    q[:, 0::2] = np.where(lo >= 8, lo - 16, lo)
    q[:, 1::2] = np.where(hi >= 8, hi - 16, hi)
    A = a.reshape(m, k).astype(np.int64)
    G = k // group
    out = np.empty(m * n, np.float32)
    for mi in range(m):
        for ni in range(n):
            acc = np.float32(0.0)
            for g in range(G):
                d = int((A[mi, g * group:(g + 1) * group] * q[ni, g * group:(g + 1) * group]).sum())
                assert -2**31 <= d < 2**31
                acc = np.float32(acc + np.float32(scales[ni * G + g] * np.float32(d)))
            out[mi * n + ni] = acc
    return out


INT4_CASES = [(1, 16, 1, 16), (1, 32, 1, 32), (2, 32, 3, 16), (3, 48, 2, 16), (4, 64, 5, 32),
              (5, 96, 7, 16), (7, 128, 6, 32), (8, 160, 9, 16), (9, 16, 4, 16), (16, 64, 13, 16),
              (17, 32, 5, 32), (33, 48, 3, 16)]


def test_packed_int4_randomized_cases(oracle):
    rng = Xs64(0x1A2B3C4D5E6F7081)
    for m, k, n, group in INT4_CASES:
        a = rng.fill_i8q(m * k)
        bp = rng.fill_bytes(n * (k // 2))
        sc = rng.fill_scales(n * (k // group))
        got = oracle.igemm_s4s8_packed(a, bp, sc, group, m, k, n)
        assert np.array_equal(got.view(np.uint32), spec_packed(a, bp, sc, group, m, k, n).view(np.uint32))


def test_packed_int4_adversarial_k6848(oracle):
    k = 6848
    for group in (16, 32):
        m, n = 4, 5
        a = np.array([127 if i % 2 == 0 else -127 for i in range(m * k)], np.int8)
        bp = np.full(n * k // 2, 0x88, np.uint8)
        sc = np.ones(n * (k // group), np.float32)
        got = oracle.igemm_s4s8_packed(a, bp, sc, group, m, k, n)
        assert np.array_equal(got, spec_packed(a, bp, sc, group, m, k, n))


# ---- src/quant tests -------------------------------------------------------

def test_int4_per_group_scales(oracle):
    w = np.zeros((1, 32), np.float32)
    w[0, 0], w[0, 16], w[0, 17] = 7.0, 14.0, -7.0
    p, s = oracle.pack_int4(w, 16)
    assert s.ravel().tolist() == [1.0, 2.0]
    codes = oracle.unpack_to_i8(p, 1, 32)
    assert (codes[0], codes[16], codes[17]) == (7, 7, -4)  # -3.5 ties-even -> -4


def test_int4_zero_group_and_clamp(oracle):
    p, s = oracle.pack_int4(np.zeros((1, 16), np.float32), 16)
    assert s.ravel().tolist() == [1.0] and (oracle.unpack_to_i8(p, 1, 16) == 0).all()
    w = np.zeros((1, 16), np.float32)
    w[0, 0], w[0, 1] = 16.0, -16.0
    p, s = oracle.pack_int4(w, 16)
    c = oracle.unpack_to_i8(p, 1, 16)
    assert (c[0], c[1]) == (7, -7)


def test_int4_pack_low_nibble_first(oracle):
    w = np.zeros((1, 16), np.float32)
    w[0, :4] = [1.0, 2.0, 7.0, -8.0]
    w[0, 4] = 8.0  # sets the group max so scale = 8/7
    p, s = oracle.pack_int4(w, 16)
    c = oracle.unpack_to_i8(p, 1, 16)
    assert (p[0, 0] & 0xF) == (c[0] & 0xF) and (p[0, 0] >> 4) == (c[1] & 0xF)


def test_int8_weight_quant_kats(oracle):
    q, s = oracle.quantize_int8_weights(np.array([[-1000.0, 1000.0]], np.float32))
    assert q.tolist() == [[-127, 127]]
    q, s = oracle.quantize_int8_weights(np.array([[254.0, -2.0, 100.0]], np.float32))
    assert s[0] == 2.0 and (q.astype(np.float32) * s[0]).tolist() == [[254.0, -2.0, 100.0]]
    q, s = oracle.quantize_int8_weights(np.array([[127.0, -127.0], [254.0, -254.0]], np.float32))
    assert s.tolist() == [1.0, 2.0] and q[0, 1] == -127
    q, s = oracle.quantize_int8_weights(np.zeros((1, 3), np.float32))
    assert s.tolist() == [1.0] and (q == 0).all()


# ---- activation quantisation (decoder.rs:1588-1597 / nn.rs:601-628) --------

def test_activation_quant_rounding(oracle):
    x = np.array([-127.0, -2.5, -1.5, -0.5, 0.5, 1.5, 2.5, 127.0], np.float32)
    q_te, s_te = oracle.quantize_row_i8(x, ties_even=True)
    q_ha, s_ha = oracle.quantize_row_i8(x, ties_even=False)
    assert s_te == s_ha == 1.0
    assert q_te.tolist() == [-127, -2, -2, 0, 0, 2, 2, 127]   # nn.rs:601-628 KAT
    assert q_ha.tolist() == [-127, -3, -2, -1, 1, 2, 3, 127]  # f32::round: half away
    q0, s0 = oracle.quantize_row_i8(np.zeros(5, np.float32))
    assert s0 == 1.0 and (q0 == 0).all()


# ---- router (native_engine/moe.rs tests :777-883) --------------------------

def _router_case(vals):
    H, E = 1280, 64
    x = np.zeros((1, H), np.float32)
    x[0, 0] = 1.0
    gate = np.zeros((E, H), np.float32)
    for e, v in vals.items():
        gate[e, 0] = v
    return x, gate


def test_route_top6_unnormalized(oracle):
    x, gate = _router_case({10: 10.0, 11: 9.0, 12: 8.0, 13: 7.0, 14: 6.0, 15: 5.0})
    rc, idx, w = oracle.route(x, gate, 6, False, 1.0)
    assert rc == 0 and idx[0].tolist() == [10, 11, 12, 13, 14, 15]
    denom = sum(math.exp(gate[e, 0]) for e in range(64))
    for j, e in enumerate(idx[0]):
        assert abs(w[0, j] - math.exp(gate[e, 0]) / denom) < 1e-5
    assert w[0].sum() < 0.9999


def test_route_renorm_and_scaling(oracle):
    x, gate = _router_case({e: 6.0 - e for e in range(6)})
    rc, idx, w = oracle.route(x, gate, 6, True, 1.0)
    assert rc == 0 and abs(float(w[0].sum()) - 1.0) < 1e-5
    assert all(w[0, j] <= w[0, j - 1] for j in range(1, 6))
    _, _, base = oracle.route(x, gate, 6, False, 1.0)
    _, _, scaled = oracle.route(x, gate, 6, False, 2.5)
    assert np.all(np.abs(scaled - 2.5 * base) < 1e-5)


def test_route_nan_is_error(oracle):
    x = np.zeros((1, 1280), np.float32)
    x[0, 0] = np.nan
    rc, _, _ = oracle.route(x, np.zeros((64, 1280), np.float32), 6, False, 1.0)
    assert rc < 0


def test_route_ties_pick_lowest_index(oracle):
    x, gate = _router_case({})  # all 64 logits equal
    rc, idx, _ = oracle.route(x, gate, 6, False, 1.0)
    assert rc == 0 and idx[0].tolist() == [0, 1, 2, 3, 4, 5]


# ---- SwiGLU hand value (moe.rs:892-915) ------------------------------------

def test_swiglu_hand_value(oracle):
    s2, sm2 = oracle.silu(2.0), oracle.silu(-2.0)
    assert abs(s2 - 1.7615942) < 1e-6 and abs(sm2 - (-0.23840584)) < 1e-6
    y = np.float32(np.float32(s2) * np.float32(6.0)) + np.float32(np.float32(sm2) * np.float32(2.0))
    assert abs(float(y) - 10.092754) < 1e-5


# ---- sampler.rs tests :618-650 and vocab tiles (decoder.rs:1851-1865) -------

@pytest.mark.parametrize("row,want", [([0.1, -2.0, 3.5, 3.4, 0.0], 2), ([0.0, 5.0, 1.0, 5.0], 1),
                                      ([float("nan"), float("-inf"), 2.0, 1.0], 2),
                                      ([float("nan")] * 3, 0)])
def test_argmax_row(oracle, row, want):
    assert oracle.argmax_row(np.array(row, np.float32)) == want


@pytest.mark.parametrize("tiles", [1, 7, 11, 1000, 200000])
def test_vocab_tile_ranges(oracle, tiles):
    n = 129280
    r = oracle.vocab_tile_ranges(n, tiles)
    assert r[0][0] == 0 and r[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
    lens = [e - s for s, e in r]
    assert max(lens) - min(lens) <= 1 and lens == sorted(lens, reverse=True)


# ---- tests/int32_overflow_proof.rs -------------------------------------------

def test_int32_boundary_k(oracle):
    """stress_k_at_the_i32_boundary (:363-424): the largest U8S8 K whose
    all-extreme dot fits i32 (66311 of 255*127) accumulates exactly; the S8S8
    cliff is K = 133144 of 127*127."""
    k = 66_311
    assert k * 255 * 127 < 2 ** 31 - 1 < (k + 1) * 255 * 127
    out = np.zeros(1, np.int32)
    oracle.igemm_u8s8(np.full(k, 255, np.uint8), np.full(k, 127, np.int8), 1, k, 1, out)
    assert int(out[0]) == k * 255 * 127
    ks = 133_144
    assert ks * 127 * 127 < 2 ** 31 - 1 < (ks + 1) * 127 * 127
    out = np.zeros(1, np.int32)
    oracle.igemm_s8s8(np.full(ks, 127, np.int8), np.full(ks, 127, np.int8), 1, ks, 1, out)
    assert int(out[0]) == ks * 127 * 127


def test_multi_channel_worst_case_accumulators(oracle):
    """multi_channel_gemm_each_accumulator_independent (:426-464): a [3, 6848]
    x [6848, 4] GEMM of extreme operands equals the i64 product cell by cell."""
    m, k, n = 3, 6848, 4
    g = np.random.default_rng(6848)
    a = g.choice(np.array([-128, 127], np.int8), size=m * k)
    b = g.choice(np.array([-128, 127], np.int8), size=n * k)
    out = np.zeros(m * n, np.int32)
    oracle.igemm_s8s8(a, b, m, k, n, out)
    assert np.array_equal(out.astype(np.int64), i64_ref(a, b, m, k, n))
