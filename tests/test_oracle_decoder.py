"""Oracle KATs for the decoder pieces beside the MoE layer, ported from the
reference's own tests: RoPE (native_engine/decoder.rs tests after :3710),
the R-SWA decode attention semantics (rswa.rs:894-944) and RMSNorm."""
import numpy as np

from oracle import oracle as O


def test_rope_position_zero_is_identity():
    c, s = O.rope_table([0], 4)
    x = np.array([[1.0, 2.0, 3.0, 4.0]], np.float32)
    assert np.array_equal(O.apply_rope(x, c, s, 4), x)


def test_rope_hand_computed_rotate_half():
    c, s = O.rope_table([1], 2)          # head_dim 2: inv_freq 1, angle = pos
    y = O.apply_rope(np.array([[3.0, 5.0]], np.float32), c, s, 2)
    sn, cs = np.sin(1.0), np.cos(1.0)
    assert abs(y[0, 0] - (3 * cs - 5 * sn)) < 1e-5
    assert abs(y[0, 1] - (5 * cs + 3 * sn)) < 1e-5


def test_rope_preserves_norm_per_head():
    c, s = O.rope_table([7, 13], 4)
    x = (np.arange(16, dtype=np.float32) * 0.25 - 2.0).reshape(2, 8)
    y = O.apply_rope(x, c, s, 4)
    n0 = (x.reshape(2, 2, 4) ** 2).sum(-1)
    n1 = (y.reshape(2, 2, 4) ** 2).sum(-1)
    assert np.all(np.abs(n0 - n1) < 1e-4)


def test_rope_heads_share_phase():
    c, s = O.rope_table([5], 4)
    x = np.array([[1.0, -2.0, 0.5, 3.0, 1.0, -2.0, 0.5, 3.0]], np.float32)
    y = O.apply_rope(x, c, s, 4)
    assert np.array_equal(y[0, :4], y[0, 4:])


def _cache(rng, heads, stride, hd):
    return rng.standard_normal((heads, stride, hd)).astype(np.float32)


def test_attention_single_key_returns_its_value():
    rng = np.random.default_rng(1)
    heads, hd = 2, 8
    q = rng.standard_normal((heads, hd)).astype(np.float32)
    k, v = _cache(rng, heads, 4, hd), _cache(rng, heads, 4, hd)
    empty = np.zeros((heads, 1, hd), np.float32)
    out = O.attention_decode(q, k, v, 1, empty, empty, 0)
    assert np.array_equal(out, v[:, 0])


def test_attention_equal_scores_average_values():
    heads, hd = 1, 4
    q = np.zeros((heads, hd), np.float32)          # every score is 0
    k = np.ones((heads, 2, hd), np.float32)
    v = np.array([[[1, 2, 3, 4], [3, 2, 1, 0]]], np.float32)
    ring_k = np.ones((heads, 2, hd), np.float32)
    ring_v = np.array([[[5, 5, 5, 5], [0, 0, 0, 0]]], np.float32)
    out = O.attention_decode(q, k, v, 2, ring_k, ring_v, 1)   # 3 keys: 2 reference + 1 ring
    want = (v[0, 0] + v[0, 1] + ring_v[0, 0]) / 3.0
    assert np.allclose(out[0], want, atol=1e-6)


def test_rms_norm_constant_row():
    c, eps = 3.0, 1e-6
    y = O.rms_norm(np.full((1, 1280), c, np.float32), eps=eps)
    assert np.allclose(y, c / np.sqrt(c * c + eps), rtol=1e-6)
    w = np.linspace(0.5, 1.5, 1280, dtype=np.float32)
    yw = O.rms_norm(np.full((1, 1280), c, np.float32), w, eps)
    assert np.array_equal(yw, (y * w).astype(np.float32))
