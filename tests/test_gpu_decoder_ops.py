"""GPU parity of the decoder pieces beside the MoE layer against the oracle:
RMSNorm and RoPE bit for bit; the R-SWA decode attention reproduces the
per-key online fold's arithmetic exactly (its exponentials are glibc's expf on
both sides), so it is bit-identical too."""
import numpy as np
import pytest

from tests.test_gpu_moe import assert_close_rel

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,cols,weighted", [(5, 1280, True), (3, 1000, False), (64, 1280, True)])
def test_rms_norm_bit_exact(cuda, rows, cols, weighted):
    import torch

    from franken_ocr_b200 import decoder_ops as D
    from oracle import oracle as O

    rng = np.random.default_rng(rows * cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32) * 3
    w = rng.uniform(0.5, 1.5, cols).astype(np.float32) if weighted else None
    want = O.rms_norm(x, w, 1e-6)
    got = D.rms_norm(x, w, 1e-6)                                   # host buffers
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    xd = torch.from_numpy(x).cuda()
    wd = torch.from_numpy(w).cuda() if weighted else None
    gd = D.rms_norm(xd, wd, 1e-6)                                  # device tensors
    torch.cuda.synchronize()
    assert np.array_equal(gd.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("positions", [list(range(7)), [0, 1, 511, 1023, 1151, 4000]])
def test_rope_bit_exact(cuda, positions):
    from franken_ocr_b200 import decoder_ops as D
    from oracle import oracle as O

    hd, heads = 128, 10
    rng = np.random.default_rng(len(positions))
    x = rng.standard_normal((len(positions), heads * hd)).astype(np.float32)
    c, s = O.rope_table(positions, hd)
    want = O.apply_rope(x, c, s, hd)
    got = D.apply_rope(x.copy(), c, s, hd)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("prefill,ring", [(1, 0), (1000, 37), (1024, 128), (0, 5), (300, 1)])
def test_attention_decode_matches_fold(cuda, prefill, ring):
    import torch

    from franken_ocr_b200 import decoder_ops as D
    from oracle import oracle as O

    heads, hd, ref_cap, W = 10, 128, 1024, 128
    rng = np.random.default_rng(prefill * 131 + ring)
    q = rng.standard_normal((heads, hd)).astype(np.float32)
    rk = rng.standard_normal((heads, ref_cap, hd)).astype(np.float32)
    rv = rng.standard_normal((heads, ref_cap, hd)).astype(np.float32)
    gk = rng.standard_normal((heads, W, hd)).astype(np.float32)
    gv = rng.standard_normal((heads, W, hd)).astype(np.float32)
    want = O.attention_decode(q, rk, rv, prefill, gk, gv, ring)
    dev = [torch.from_numpy(a).cuda() for a in (q, rk, rv, gk, gv)]
    got = D.attention_decode(dev[0], dev[1], dev[2], prefill, dev[3], dev[4], ring)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    if prefill + ring == 1:
        src = rv if prefill else gv
        assert np.array_equal(got, src[:, 0])                      # one key: its value
    else:
        assert_close_rel(got, want, f"attention {prefill}+{ring}")
