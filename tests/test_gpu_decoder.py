"""GPU parity of the config-3 decoder: the new ops against the oracle
(bit-exact for the int8 projections, SwiGLU and residual add; causal prefill
attention in the oracle's evaluation order, bit-exact: exp is glibc's expf on
both sides), then whole decoders: prefill, R-SWA
decode steps through a ring wrap, and identical greedy tokens."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.mark.parametrize("m", [1, 5, 16, 17, 64, 200])
@pytest.mark.parametrize("te", [False, True])
def test_linear_i8_bit_exact(cuda, oracle, m, te):
    import torch

    from franken_ocr_b200._lib import MEM_DEVICE, check, lib

    g = np.random.default_rng(100 + m)
    K, N = 1280, 1280 + 256
    x = g.standard_normal((m, K), dtype=np.float32)
    w = g.integers(-127, 128, (N, K), dtype=np.int8)
    ws = g.uniform(0.001, 0.02, N).astype(np.float32)
    want = oracle.linear_i8(x, w, ws, te)
    # host mode
    y = np.empty((m, N), np.float32)
    check(lib.focr_linear_i8(x.ctypes.data, m, K, w.ctypes.data, ws.ctypes.data, N, int(te),
                             y.ctypes.data, 0, None))
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
    # device mode
    dx, dw, ds = (torch.from_numpy(a).cuda() for a in (x, w, ws))
    dy = torch.empty((m, N), dtype=torch.float32, device="cuda")
    check(lib.focr_linear_i8(dx.data_ptr(), m, K, dw.data_ptr(), ds.data_ptr(), N, int(te),
                             dy.data_ptr(), MEM_DEVICE, torch.cuda.current_stream().cuda_stream))
    assert np.array_equal(dy.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_swiglu_and_add_bit_exact(cuda, oracle):
    from franken_ocr_b200._lib import check, lib

    g = np.random.default_rng(7)
    rows, inter = 3, 1001
    gu = (g.standard_normal((rows, 2 * inter), dtype=np.float32) * 4).astype(np.float32)
    act = np.empty((rows, inter), np.float32)
    check(lib.focr_swiglu(gu.ctypes.data, rows, inter, act.ctypes.data, 0, None))
    want = np.array([[oracle.silu(float(gu[r, i])) * gu[r, inter + i] for i in range(inter)]
                     for r in range(rows)], np.float32)
    # silu's exp is glibc's expf on both sides: bit-exact
    assert np.array_equal(act.view(np.uint32), want.view(np.uint32))
    a = g.standard_normal(1283, dtype=np.float32)
    b = g.standard_normal(1283, dtype=np.float32)
    y = np.empty_like(a)
    check(lib.focr_add(a.ctypes.data, b.ctypes.data, a.size, y.ctypes.data, 0, None))
    assert np.array_equal(y, a + b)


@pytest.mark.parametrize("seq", [1, 31, 33, 100, 300])
def test_attention_prefill_close(cuda, oracle, seq):
    from franken_ocr_b200._lib import check, lib

    g = np.random.default_rng(seq)
    heads = 10
    q, k, v = (g.standard_normal((seq, heads * 128), dtype=np.float32) for _ in range(3))
    out = np.empty_like(q)
    check(lib.focr_attention_prefill(q.ctypes.data, k.ctypes.data, v.ctypes.data, seq, heads,
                                     128, out.ctypes.data, 0, None))
    want = oracle.attention_prefill(q, k, v, heads)
    from tests.test_gpu_moe import assert_close_rel

    assert_close_rel(out, want, f"prefill attention seq={seq}")
    assert np.array_equal(out[0], v[0])


def _run_decoder(oracle, W, seq, n_tokens, seed):
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.decoder import DecoderI8

    e = synth.prompt_embeds(seed, seq, W.hidden)
    O = oracle.DecoderOracle(W)
    hid = []
    want = O.generate(e, n_tokens, hiddens=hid)
    D = DecoderI8(W, max_prefill=seq)
    h = D.prefill(torch.from_numpy(e).cuda())
    got, errs = [], []
    for i in range(n_tokens):
        errs.append(rel_err(h[-1].cpu().numpy(), hid[i]))
        _, bi = D.lm_head_top1(h[-1:])
        tok = int(bi.item())
        got.append(tok)
        if i + 1 < n_tokens:
            h = D.decode_step(D.embed[tok:tok + 1], seq + i)
    D.close()
    return np.array(got), want, errs


def test_small_decoder_greedy_tokens_through_ring_wrap(cuda, oracle):
    """3 layers (dense + 2 MoE of 8 experts), 40-token prefill, 140 greedy
    tokens: the 128-slot ring fills and wraps."""
    from franken_ocr_b200 import synth

    W = synth.decoder_model(11, layers=3, n_experts=8, dense_inter=512, vocab=2048)
    got, want, errs = _run_decoder(oracle, W, 40, 140, 11)
    assert np.array_equal(got, want), np.nonzero(got != want)[0][:5]
    assert max(errs) == 0.0, max(errs)   # hidden rows bit-identical


def test_full_dims_decoder_greedy_tokens(cuda, oracle):
    """The configuration's dimensions (12 layers, 64 experts top-6 + shared,
    dense 6848, vocab 129280) on a 64-token prefill and 8 greedy tokens."""
    from franken_ocr_b200 import synth

    W = synth.decoder_model(12)
    got, want, errs = _run_decoder(oracle, W, 64, 8, 12)
    assert np.array_equal(got, want)
    assert max(errs) == 0.0, max(errs)   # hidden rows bit-identical


def test_graph_greedy_decode_matches_oracle(cuda, oracle):
    """The device-state decode step replayed from one CUDA graph gives the
    oracle's tokens through a ring wrap, and equals the eager loop; a second
    call reuses the captured graph."""
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.decoder import DecoderI8

    W = synth.decoder_model(11, layers=3, n_experts=8, dense_inter=512, vocab=2048)
    e = synth.prompt_embeds(11, 40, W.hidden)
    want = oracle.DecoderOracle(W).generate(e, 140)
    D = DecoderI8(W, max_prefill=40)
    de = torch.from_numpy(e).cuda()
    got = D.generate_graph(de, 140)
    assert np.array_equal(got, want), np.nonzero(got != want)[0][:5]
    assert (D.ring_len, D.ring_pos) == (128, 139 % 128)
    assert np.array_equal(D.generate_graph(de, 140), want)
    assert np.array_equal(D.generate_graph(de, 140, use_graph=False), want)
    assert np.array_equal(D.generate(de, 140), want)
    D.close()


def _golden_config3():
    import json
    from pathlib import Path

    return json.loads((Path(__file__).parent / "golden" / "decoder_config3_greedy256.json").read_text())


def test_config3_greedy256_matches_oracle_golden(cuda):
    """The north-star correctness bar at its stated size: the config-3 decoder
    (12 layers, seed 3), a 1024-token prefill, then 256 greedy tokens replayed
    from the captured decode graph -- every token equal to the scalar CPU
    oracle's (tests/golden/make_decoder_golden.py)."""
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.decoder import DecoderI8

    g = _golden_config3()
    W = synth.decoder_model(g["seed"])
    e = torch.from_numpy(synth.prompt_embeds(g["seed"], g["prefill_tokens"])).cuda()
    D = DecoderI8(W, max_prefill=g["prefill_tokens"])
    got = [int(t) for t in D.generate_graph(e, g["n_tokens"])]
    D.close()
    bad = [i for i, (a, b) in enumerate(zip(got, g["tokens"])) if a != b]
    assert not bad, f"first mismatch at token {bad[:1]}: {got[bad[0]]} != {g['tokens'][bad[0]]}"


def test_config3_hidden_states_equal_oracle_golden(cuda):
    """Eager decode of the same model: the final hidden row each of the first
    12 tokens is read from is bit-identical to the oracle's (its f64 sum and
    L2 norm, computed the same way from the f32 row, are equal); tokens equal."""
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.decoder import DecoderI8

    g = _golden_config3()
    W = synth.decoder_model(g["seed"])
    e = torch.from_numpy(synth.prompt_embeds(g["seed"], g["prefill_tokens"])).cuda()
    D = DecoderI8(W, max_prefill=g["prefill_tokens"])
    h = D.prefill(e)
    seq = g["prefill_tokens"]
    for i in range(12):
        row = h[-1].double().cpu().numpy()
        l2 = float(np.sqrt((row * row).sum()))
        assert l2 == g["hidden_l2"][i], (i, l2, g["hidden_l2"][i])
        assert float(row.sum()) == g["hidden_sum"][i], i
        _, bi = D.lm_head_top1(h[-1:])
        tok = int(bi.item())
        assert tok == g["tokens"][i], i
        h = D.decode_step(D.embed[tok:tok + 1], seq + i)
    D.close()
