"""The oracle's prefill MoE block (moe_block_i8, decoder.rs:2142-2181)
against an independent numpy composition of the same steps from the
oracle's pinned primitives: ties-even row quantisation (:1647-1656), the
int8 GEMV dequant ((f32)acc * a_scale) * w_scale, silu, the per-expert
ascending loop with `out[t] += w * y`, then the shared expert."""
import numpy as np

from oracle import oracle as O
from oracle.oracle import MoeOracle


def _gemv(aq, a_scale, w, ws):
    acc = (w.astype(np.int64) @ aq.astype(np.int64)).astype(np.int32)
    return (acc.astype(np.float32) * np.float32(a_scale)) * ws


def _expert_te(x, gw, gs, uw, us, dw, ds):
    xq, xs = O.quantize_row_i8(x, ties_even=True)
    g = _gemv(xq, xs, gw, gs)
    u = _gemv(xq, xs, uw, us)
    act = np.array([O.silu(float(v)) for v in g], np.float32) * u
    aq, a2 = O.quantize_row_i8(act, ties_even=True)
    return _gemv(aq, a2, dw, ds)


def test_prefill_block_matches_composition():
    from franken_ocr_b200 import synth

    H, I, E, K, S, m = 64, 32, 8, 2, 48, 7
    W = synth.moe_layer(77, hidden=H, inter=I, n_experts=E, topk=K, shared_inter=S)
    x = synth.hidden_states(78, m, hidden=H)
    idx, w = synth.zipf_routing(78, m, n_experts=E, topk=K)
    A = W.arrays
    want = np.zeros((m, H), np.float32)
    for e in range(E):
        for t in range(m):
            for j in range(K):
                if idx[t, j] != e:
                    continue
                y = _expert_te(x[t], A["gate_w"][e], A["gate_s"][e], A["up_w"][e], A["up_s"][e],
                               A["down_w"][e], A["down_s"][e])
                want[t] = want[t] + np.float32(w[t, j]) * y
    for t in range(m):
        want[t] = want[t] + _expert_te(x[t], A["sh_gate_w"], A["sh_gate_s"], A["sh_up_w"],
                                       A["sh_up_s"], A["sh_down_w"], A["sh_down_s"])
    got = MoeOracle(W).prefill_routed(x, idx, w)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
