"""Config 4 at its stated sizes: the int4 g32 MoE layer at M = 1 and M = 256
(decode semantics; the oracle's expert_s4 driver) and the int4 g32 lm-head
shard [16160, 1280] (logits = packed int4 GEMM of the quantised row times the
activation scale) with its top-1, bit-identical to the oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m", [1, 256])
def test_config4_int4_moe_layer(cuda, oracle, m):
    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer
    from oracle.oracle import MoeOracle

    W = synth.moe_layer(4400, group=32)
    L = MoeLayer(W, max_tokens=m)
    x = synth.hidden_states(4401, m)
    y, idx, w = L.decode(x)
    rc, oy, oi, ow = MoeOracle(W).decode(x)
    assert rc == 0
    assert np.array_equal(idx, oi)
    assert np.array_equal(w.view(np.uint32), ow.view(np.uint32))
    assert np.array_equal(y.view(np.uint32), oy.view(np.uint32))
    L.close()


@pytest.mark.parametrize("m,g,rows", [(1, 32, 16160), (256, 32, 16160), (1, 16, 4099)])
def test_config4_int4_lmhead_shard(cuda, oracle, m, g, rows):
    import torch

    from franken_ocr_b200.lmhead import LmHeadShard
    from franken_ocr_b200.quant import pack_int4_f32
    from franken_ocr_b200 import synth

    H = 1280
    wf = synth.normal(4402, "lm_head", 3, (rows, H), 0.02)
    packed, sc = pack_int4_f32(wf, g)
    x = synth.hidden_states(4403, m)
    head = LmHeadShard(packed, sc, row_begin=3 * rows, max_tokens=m, group=g)
    bv, bi, lg = head.top1(torch.from_numpy(x).cuda(), want_logits=True)
    torch.cuda.synchronize()
    for r in range(m):
        q, s = oracle.quantize_row_i8(x[r])
        want = oracle.igemm_s4s8_packed(q, packed.reshape(-1), sc.reshape(-1), g, 1, H, rows)
        want = (want * np.float32(s)).astype(np.float32)
        assert np.array_equal(lg[r].cpu().numpy().view(np.uint32), want.view(np.uint32)), r
        t = oracle.argmax_row(want)
        assert int(bi[r].item()) == 3 * rows + t and float(bv[r].item()) == float(want[t])
    head.close()
