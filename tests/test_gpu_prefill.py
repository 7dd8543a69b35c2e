"""GPU parity of the prefill MoE block (focr_moe_prefill, moe_block_i8 of
decoder.rs:2142-2181) against the oracle: identical routing, f32 within
1e-5 relative, on the tensor-core path, the GEMV-grouped path and int4
experts."""
import numpy as np
import pytest

from tests.test_gpu_moe import assert_close_rel

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["tc", "gemv", "int4"])
@pytest.mark.parametrize("m", [1, 33, 200])
def test_prefill_matches_oracle(cuda, oracle, monkeypatch, kind, m):
    from franken_ocr_b200 import synth
    from franken_ocr_b200.moe import MoeLayer
    from oracle.oracle import MoeOracle

    if kind == "gemv":
        monkeypatch.setenv("FOCR_DISABLE_TC", "1")
    W = synth.moe_layer(5000 + m, shared_inter=1792 if kind != "int4" else 896,
                        group=32 if kind == "int4" else 0)
    L = MoeLayer(W, max_tokens=m)
    x = synth.hidden_states(700 + m, m)
    y, idx, w = L.prefill(x)
    rc, oy, oi, ow = MoeOracle(W).prefill(x)
    assert rc == 0
    assert np.array_equal(idx, oi)
    assert_close_rel(y, oy, f"prefill {kind} m={m}")
    L.close()
