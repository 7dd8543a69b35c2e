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


# -- config-3 decoder pieces -----------------------------------------------------
def test_attention_prefill_matches_float64_softmax(oracle):
    g = np.random.default_rng(31)
    seq, heads, hd = 37, 3, 128
    q, k, v = (g.standard_normal((seq, heads * hd), dtype=np.float32) for _ in range(3))
    out = oracle.attention_prefill(q, k, v, heads, hd)
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        s = (q[:, sl].astype(np.float64) @ k[:, sl].astype(np.float64).T) / np.sqrt(hd)
        s[np.triu_indices(seq, 1)] = -np.inf
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        ref = p @ v[:, sl].astype(np.float64)
        np.testing.assert_allclose(out[:, sl], ref, rtol=1e-4, atol=1e-5)
    # causality: row t ignores keys after t; row 0 is v[0]
    assert np.array_equal(out[0], v[0])


def test_linear_i8_rows_are_gemv_and_quantised_gemm(oracle):
    g = np.random.default_rng(32)
    x = g.standard_normal((5, 96), dtype=np.float32)
    w = g.integers(-127, 128, (40, 96), dtype=np.int8)
    ws = g.uniform(0.001, 0.02, 40).astype(np.float32)
    half = oracle.linear_i8(x, w, ws, False)
    for r in range(5):
        assert np.array_equal(half[r], oracle.gemv_i8(x[r], w, ws))
    te = oracle.linear_i8(x, w, ws, True)
    for r in range(5):
        xq, s = oracle.quantize_row_i8(x[r], ties_even=True)
        acc = xq.astype(np.int64) @ w.astype(np.int64).T
        want = ((acc.astype(np.float32) * s).astype(np.float32) * ws).astype(np.float32)
        assert np.array_equal(te[r], want)


def test_swiglu_mlp_decode_row_is_expert_i8(oracle):
    from franken_ocr_b200 import synth

    W = synth.decoder_model(3, layers=1, dense_inter=256, vocab=64)
    d = W.layers[0].dense
    x = synth.prompt_embeds(3, 2)
    y = oracle.swiglu_mlp_i8(x, d, False)
    for r in range(2):
        want = oracle.expert_i8(x[r], d["gate_w"], d["gate_s"], d["up_w"], d["up_s"],
                                d["down_w"], d["down_s"])
        assert np.array_equal(y[r], want)


def test_product_rope_table_matches_oracle(oracle):
    """The product's host RopeTable builder (libfocr_cuda.so) equals the
    oracle's bit for bit over every position of a 32k context."""
    from franken_ocr_b200.decoder import rope_table

    pos = np.arange(32768)
    c, s = rope_table(pos)
    oc, os_ = oracle.rope_table(pos, 128)
    assert np.array_equal(c.view(np.uint32), oc.view(np.uint32))
    assert np.array_equal(s.view(np.uint32), os_.view(np.uint32))


def test_decoder_oracle_ring_wraps_and_is_deterministic(oracle):
    from franken_ocr_b200 import synth

    W = synth.decoder_model(5, layers=2, n_experts=4, topk=2, dense_inter=128, vocab=256,
                            shared_inter=0)
    O = oracle.DecoderOracle(W)
    e = synth.prompt_embeds(5, 6)
    t1 = O.generate(e, 131)
    assert O.ring_len == 128 and O.ring_pos == 2
    t2 = oracle.DecoderOracle(W).generate(e, 131)
    assert np.array_equal(t1, t2)
    assert t1.min() >= 0 and t1.max() < 256


def test_threaded_cpu_decoder_matches_scalar_oracle(oracle):
    """The timed CPU baseline (dispatched-tier projections, threaded MoE
    driver) gives the scalar oracle's hidden states and tokens exactly."""
    from franken_ocr_b200 import synth

    W = synth.decoder_model(6, layers=2, n_experts=8, dense_inter=256, vocab=512,
                            shared_inter=256)
    e = synth.prompt_embeds(6, 7, W.hidden)
    h1, h2 = [], []
    t1 = oracle.DecoderOracle(W).generate(e, 6, hiddens=h1)
    t2 = oracle.DecoderOracle(W, threads=4).generate(e, 6, hiddens=h2)
    assert np.array_equal(t1, t2)
    for a, b in zip(h1, h2):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
