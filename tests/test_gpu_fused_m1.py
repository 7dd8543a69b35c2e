"""GPU parity of the fused single-token MoE decode kernel (focr_moe_decode
with m == 1): one persistent launch doing router, top-k, gate+up+SwiGLU,
requantisation, down and the slot-ordered combine (decoder.rs:2199-2268).

Every case is checked against the oracle and, bit for bit, against the
multi-launch path (FOCR_DISABLE_FUSED_M1 at layer creation)."""
import numpy as np
import pytest

from tests.test_gpu_moe import assert_close_rel

pytestmark = pytest.mark.gpu


def _run(layer, xs, monkeypatch, fused):
    from franken_ocr_b200.moe import MoeLayer

    if fused:
        monkeypatch.delenv("FOCR_DISABLE_FUSED_M1", raising=False)
    else:
        monkeypatch.setenv("FOCR_DISABLE_FUSED_M1", "1")
    L = MoeLayer(layer, max_tokens=1)
    out = [L.decode(x) for x in xs]
    L.close()
    monkeypatch.delenv("FOCR_DISABLE_FUSED_M1", raising=False)
    return out


@pytest.mark.parametrize("shape", [
    dict(),                                              # config 0: 64 experts, top-6
    dict(shared_inter=1792),                             # + shared expert (configs 2/3)
    dict(hidden=64, inter=32, n_experts=16, topk=4, shared_inter=48),
    dict(hidden=208, inter=80, n_experts=40, topk=8),    # ragged per-CTA ranges
])
def test_fused_m1_matches_oracle_and_unfused(cuda, oracle, monkeypatch, shape):
    from franken_ocr_b200 import synth
    from oracle.oracle import MoeOracle

    layer = synth.moe_layer(4321, **shape)
    xs = [synth.hidden_states(300 + s, 1, hidden=layer.hidden) for s in range(3)]
    fused = _run(layer, xs, monkeypatch, True)
    plain = _run(layer, xs, monkeypatch, False)
    O = MoeOracle(layer)
    for x, (y, idx, w), (py, pidx, pw) in zip(xs, fused, plain):
        rc, oy, oi, ow = O.decode(x)
        assert rc == 0
        assert np.array_equal(idx, oi)
        assert_close_rel(y, oy, "fused m=1")
        assert np.array_equal(idx, pidx)
        assert np.array_equal(y.view(np.uint32), py.view(np.uint32))
        assert np.array_equal(w.view(np.uint32), pw.view(np.uint32))


def test_fused_m1_many_calls(cuda, oracle):
    """Grid barriers reset themselves: 200 back-to-back calls on one handle."""
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer
    from oracle.oracle import MoeOracle

    layer = synth.moe_layer(1234, shared_inter=1792)
    L = MoeLayer(layer, max_tokens=1)
    x = synth.hidden_states(77, 1)
    xd = torch.from_numpy(x).cuda()
    ys = [L.decode(xd)[0].clone() for _ in range(200)]
    torch.cuda.synchronize()
    rc, oy, _, _ = MoeOracle(layer).decode(x)
    for y in ys[::37] + [ys[-1]]:
        assert_close_rel(y.cpu().numpy(), oy, "fused repeated")
    assert all(torch.equal(ys[0], y) for y in ys)
    L.close()
