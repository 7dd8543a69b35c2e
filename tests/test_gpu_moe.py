"""GPU parity of the MoE decode layer and the lm-head against the oracle.

Bars (the north star's): identical top-6 expert selection, f32 outputs within
1e-5 relative, identical greedy tokens -- and beyond them, bit-identical f32
outputs: every f32 step follows the reference's order with separately rounded
operations, and exp is glibc's expf on both sides, so assert_close_rel checks
the 1e-5 bound and then requires every element to match bit for bit.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def assert_close_rel(got, want, what, min_exact=1.0):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    scale = np.sqrt(np.mean(want.astype(np.float64) ** 2, axis=-1, keepdims=True)) + 1e-30
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    bound = RTOL * (np.abs(want.astype(np.float64)) + scale)
    assert np.all(err <= bound), f"{what}: max err/bound {np.max(err / bound):.3g}"
    exact = np.mean(got.view(np.uint32) == want.view(np.uint32))
    assert exact >= min_exact, f"{what}: only {exact:.4f} bit-exact"
    return exact


@pytest.fixture(scope="module")
def layer0():
    from franken_ocr_b200 import synth

    return synth.moe_layer(1234)          # config 0: 64 experts, top-6, no shared


@pytest.fixture(scope="module")
def layer2():
    from franken_ocr_b200 import synth

    return synth.moe_layer(99, shared_inter=1792)   # configs 2/3: + fused shared expert


def test_router_kats_on_gpu(cuda, oracle):
    """moe.rs:777-883 hand cases through the GPU router."""
    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer

    W = synth.moe_layer(5, n_experts=64, inter=32, hidden=1280)
    W.router = np.zeros((64, 1280), np.float32)
    for e, v in {10: 10.0, 11: 9.0, 12: 8.0, 13: 7.0, 14: 6.0, 15: 5.0}.items():
        W.router[e, 0] = v
    x = np.zeros((3, 1280), np.float32)
    x[:, 0] = 1.0
    for norm in (False, True):
        L = MoeLayer(W, max_tokens=3, norm_topk_prob=norm)
        idx, w = L.route(x)
        rc, oi, ow = oracle.route(x, W.router, 6, norm, 1.0)
        assert rc == 0 and idx.tolist() == oi.tolist()
        assert idx[0].tolist() == [10, 11, 12, 13, 14, 15]
        assert np.array_equal(w.view(np.uint32), ow.view(np.uint32))
        if norm:
            assert abs(float(w[0].sum()) - 1.0) < 1e-5
        L.close()
    # all-equal logits: ties go to the lowest index
    W.router[:] = 0.0
    L = MoeLayer(W, max_tokens=3)
    idx, _ = L.route(x)
    assert idx[0].tolist() == [0, 1, 2, 3, 4, 5]
    # NaN input: the reference's "no finite router score" error
    xn = x.copy()
    xn[0, 0] = np.nan
    from franken_ocr_b200._lib import FOCR_E_ROUTE, FocrError

    with pytest.raises(FocrError) as ei:
        L.route(xn)
    assert ei.value.code == FOCR_E_ROUTE
    L.close()


@pytest.mark.parametrize("m", [1, 3, 16])
def test_route_matches_oracle(cuda, oracle, layer0, m):
    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer

    L = MoeLayer(layer0, max_tokens=m)
    x = synth.hidden_states(7, m)
    idx, w = L.route(x)
    rc, oi, ow = oracle.route(x, layer0.router, 6, True, 1.0)
    assert rc == 0
    assert np.array_equal(idx, oi)
    assert_close_rel(w, ow, "router weights")
    L.close()


@pytest.mark.parametrize("m", [1, 2, 5])
def test_decode_config0(cuda, oracle, layer0, m):
    """Config 0: one MoE layer, decode, top-6 renormalised, no shared expert."""
    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer
    from oracle.oracle import MoeOracle

    L = MoeLayer(layer0, max_tokens=m)
    O = MoeOracle(layer0, norm_topk_prob=True)
    for step in range(2):
        x = synth.hidden_states(11 + step, m)
        y, idx, w = L.decode(x)
        rc, oy, oi, ow = O.decode(x)
        assert rc == 0
        assert np.array_equal(idx, oi)
        assert_close_rel(y, oy, f"decode m={m}")
    L.close()


def test_forward_config2_zipf(cuda, oracle, layer2):
    """Config 2: 64 sequences, Zipf(1.1) routing, + fused shared expert."""
    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer
    from oracle.oracle import MoeOracle

    m = 64
    L = MoeLayer(layer2, max_tokens=m)
    O = MoeOracle(layer2)
    x = synth.hidden_states(21, m)
    idx, w = synth.zipf_routing(21, m)
    y = L.forward(x, idx, w)
    assert_close_rel(y, O.forward(x, idx, w), "forward m=64 zipf")
    L.close()


def test_decode_device_tensors(cuda, oracle, layer2):
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer
    from oracle.oracle import MoeOracle

    m = 4
    L = MoeLayer(layer2, max_tokens=m)
    x = synth.hidden_states(31, m)
    xd = torch.from_numpy(x).cuda()
    y, idx, w = L.decode(xd)
    torch.cuda.synchronize()
    rc, oy, oi, ow = MoeOracle(layer2).decode(x)
    assert np.array_equal(idx.cpu().numpy(), oi)
    assert_close_rel(y.cpu().numpy(), oy, "device decode")
    L.close()


def test_lmhead_shards_and_argmax(cuda, oracle):
    """Vocab shards (8 x 16160) reproduce the monolithic head's logits and
    argmax (tests/lmhead_shard_parity.rs at the real [129280, 1280] shape)."""
    from franken_ocr_b200 import synth
    from franken_ocr_b200.lmhead import LmHeadShard, top1_combine

    V, H, m = 129280, 1280, 3
    q, s = synth.lm_head(17, V)
    x = synth.hidden_states(41, m)
    full = LmHeadShard(q, s, 0, max_tokens=m)
    fv, fi, flog = full.top1(x, want_logits=True)
    for r in range(m):
        want = oracle.gemv_i8(x[r], q, s)
        assert np.array_equal(flog[r].view(np.uint32), want.view(np.uint32))
        assert fi[r] == oracle.argmax_row(want)
    vals, idxs = [], []
    for sh in range(8):
        lo = sh * 16160
        shard = LmHeadShard(q[lo:lo + 16160], s[lo:lo + 16160], lo, max_tokens=m)
        v, i, lg = shard.top1(x, want_logits=True)
        assert np.array_equal(lg.view(np.uint32), flog[:, lo:lo + 16160].view(np.uint32))
        vals.append(v)
        idxs.append(i)
        shard.close()
    tok = top1_combine(np.stack(vals), np.stack(idxs))
    assert tok.tolist() == fi.astype(np.uint32).tolist()
    full.close()


def test_forward_gemv_grouped_path(cuda, oracle, layer2, monkeypatch):
    """The dp4a GEMV-grouped expert kernels (used when the tensor-core path is
    disabled or the shapes are not multiples of 128) at m = 64."""
    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer
    from oracle.oracle import MoeOracle

    monkeypatch.setenv("FOCR_DISABLE_TC", "1")
    m = 64
    L = MoeLayer(layer2, max_tokens=m)
    x = synth.hidden_states(22, m)
    idx, w = synth.zipf_routing(22, m)
    y = L.forward(x, idx, w)
    assert_close_rel(y, MoeOracle(layer2).forward(x, idx, w), "gemv-grouped forward m=64")
    L.close()


@pytest.mark.parametrize("m", [2, 17, 128, 300])
def test_forward_tc_token_counts(cuda, oracle, m):
    """Tensor-core expert path across token counts, incl. experts with more
    than 128 tokens (several N jobs per CTA) and uniform routing."""
    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer
    from oracle.oracle import MoeOracle

    W = synth.moe_layer(77, n_experts=8, shared_inter=256, inter=256)
    L = MoeLayer(W, max_tokens=m)
    x = synth.hidden_states(m, m)
    idx, w = synth.zipf_routing(m, m, n_experts=8)
    y = L.forward(x, idx, w)
    assert_close_rel(y, MoeOracle(W).forward(x, idx, w), f"tc forward m={m}")
    L.close()


@pytest.mark.parametrize("m", [3, 64, 300])
def test_forward_fused_launch(cuda, oracle, monkeypatch, m):
    """The single persistent launch (FOCR_MOE_FUSED=1: gate+up, last-arriver
    requantisation per expert, down) gives the same bits as the oracle."""
    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer
    from oracle.oracle import MoeOracle

    monkeypatch.setenv("FOCR_MOE_FUSED", "1")
    W = synth.moe_layer(811, shared_inter=1792)
    L = MoeLayer(W, max_tokens=m)
    x = synth.hidden_states(812, m)
    idx, w = synth.zipf_routing(812, m)
    y = L.forward(x, idx, w)
    want = MoeOracle(W).forward(x, idx, w)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
    L.close()


@pytest.mark.parametrize("path", ["fusedq", "fused2"])
@pytest.mark.parametrize("m", [2, 64, 300])
def test_forward_fusedq_launch(cuda, oracle, monkeypatch, m, path):
    """The single persistent launches -- on-load requantisation
    (FOCR_MOE_PATH=fusedq: the down GEMM's producer warps quantise the act rows
    with the gate+up epilogue's per-row maximum) and split B loads
    (fused2: weights never wait, one warp loads each down job's act rows once
    its expert is requantised) -- give the same bits as the oracle, for decode
    (forward) and prefill (ties-even) semantics, twice in a row on one
    handle."""
    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer
    from oracle.oracle import MoeOracle

    monkeypatch.setenv("FOCR_MOE_PATH", path)
    W = synth.moe_layer(813, shared_inter=1792)
    L = MoeLayer(W, max_tokens=m)
    O = MoeOracle(W)
    for step in range(2):
        x = synth.hidden_states(814 + step, m)
        idx, w = synth.zipf_routing(814 + step, m)
        y = L.forward(x, idx, w)
        want = O.forward(x, idx, w)
        assert np.array_equal(y.view(np.uint32), want.view(np.uint32)), step
    x = synth.hidden_states(820, m)
    y, _, _ = L.prefill(x)
    _, want, _, _ = O.prefill(x)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
    L.close()
