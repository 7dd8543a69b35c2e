"""The library-side decoder (focr_decoder_*, DecoderLib): weights, caches,
activation buffers and the captured decode graph all owned by
libfocr_cuda.so, host numpy in and out -- the path a host without PyTorch
drives.  Checked against the CPU oracle and the config-3 golden tokens."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_decoder_lib_small_greedy_through_ring_wrap(cuda, oracle):
    """3 layers (dense + 2 MoE of 8 experts), 40-token prefill, 140 greedy
    tokens through the ring wrap: the oracle's tokens; the prefill hidden
    states equal the per-op driver's bit for bit; a second call (captured
    graph reused) and a shorter one (re-captured) agree."""
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.decoder import DecoderI8, DecoderLib

    W = synth.decoder_model(11, layers=3, n_experts=8, dense_inter=512, vocab=2048)
    e = synth.prompt_embeds(11, 40, W.hidden)
    want = oracle.DecoderOracle(W).generate(e, 140)
    D = DecoderLib(W, max_prefill=40)
    got = D.generate(e, 140)
    assert np.array_equal(got, want), np.nonzero(got != want)[0][:5]
    assert np.array_equal(D.generate(e, 140), want)
    assert np.array_equal(D.generate(e, 17), want[:17])
    h_lib = D.prefill(e)
    P = DecoderI8(W, max_prefill=40)
    h_ops = P.prefill(torch.from_numpy(e).cuda()).cpu().numpy()
    P.close()
    assert np.array_equal(h_lib.view(np.uint32), h_ops.view(np.uint32))
    D.close()


def test_decoder_lib_rejects_bad_shapes(cuda):
    from franken_ocr_b200 import synth
    from franken_ocr_b200._lib import FocrError
    from franken_ocr_b200.decoder import DecoderLib

    W = synth.decoder_model(12, layers=2, n_experts=8, dense_inter=256, vocab=512)
    D = DecoderLib(W, max_prefill=8)
    with pytest.raises(FocrError):
        D.prefill(synth.prompt_embeds(12, 9, W.hidden))
    D.close()


def test_decoder_lib_config3_greedy256_matches_golden(cuda):
    """The north-star bar through the library decoder: config 3 (12 layers,
    seed 3), 1024-token prefill, 256 greedy tokens equal to the scalar CPU
    oracle's (tests/golden/decoder_config3_greedy256.json)."""
    import json
    from pathlib import Path

    from franken_ocr_b200 import synth
    from franken_ocr_b200.decoder import DecoderLib

    g = json.loads((Path(__file__).parent / "golden" / "decoder_config3_greedy256.json").read_text())
    W = synth.decoder_model(g["seed"])
    e = synth.prompt_embeds(g["seed"], g["prefill_tokens"])
    D = DecoderLib(W, max_prefill=g["prefill_tokens"])
    got = [int(t) for t in D.generate(e, g["n_tokens"])]
    D.close()
    bad = [i for i, (a, b) in enumerate(zip(got, g["tokens"])) if a != b]
    assert not bad, f"first mismatch at token {bad[:1]}"
