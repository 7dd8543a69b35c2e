"""GPU engine loaded from a ``.focrq`` file: a layer written with the
deterministic writer, read back by the validating reader and uploaded through
``focr_moe_create`` decodes bit-identically to the oracle on the arrays that
were written (int8 and int4 experts), and an lm-head shard read from the same
file gives the oracle's greedy token."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("group,shared", [(0, 1792), (32, 0)])
def test_moe_layer_from_focrq(cuda, oracle, tmp_path, group, shared):
    from franken_ocr_b200 import focrq, synth
    from franken_ocr_b200.moe import MoeLayer
    from oracle.oracle import MoeOracle

    W = synth.moe_layer(4200 + group, shared_inter=shared, group=group)
    wr = focrq.Writer(source_sha256=focrq.sha256_bytes(b"synthetic"))
    focrq.write_moe_layer(wr, 2, W)
    path = tmp_path / "layer.focrq"
    wr.write(path)
    L = MoeLayer(focrq.moe_layer_weights(focrq.Weights.load(path), 2), max_tokens=4)
    O = MoeOracle(W)
    x = synth.hidden_states(610, 4)
    _, oy, oi, ow = O.decode(x)
    yf = L.forward(x, oi, ow)
    assert np.array_equal(yf.view(np.uint32), oy.view(np.uint32))
    _, idx, _ = L.decode(x)
    assert np.array_equal(idx, oi)
    L.close()


def test_lm_head_shard_from_focrq(cuda, oracle, tmp_path):
    from franken_ocr_b200 import focrq, synth
    from franken_ocr_b200.lmhead import LmHeadShard
    from oracle.oracle import argmax_row, gemv_i8

    q, s = synth.lm_head(9, 16160)
    wr = focrq.Writer()
    wr.add_qint8("lm_head.weight", q, s)
    path = tmp_path / "head.focrq"
    wr.write(path)
    w = focrq.Weights.load(path)
    qs, ss = focrq.lm_head_weights(w, 8080, 8080)
    H = LmHeadShard(qs, ss, row_begin=8080)
    x = synth.hidden_states(611, 1)
    bv, bi, lg = H.top1(x, want_logits=True)
    want = gemv_i8(x[0], qs, ss)
    assert np.array_equal(lg[0].view(np.uint32), want.view(np.uint32))
    assert bi[0] == 8080 + argmax_row(want)
    H.close()
