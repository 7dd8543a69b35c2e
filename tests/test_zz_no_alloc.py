"""focr_gemv_i8_noalloc: the dequant GEMV for callers that cannot allocate
device memory (an embedder whose GPU memory is owned by its own pool
allocator, or code where an allocation would block or is not allowed).

It must give the same result as focr_gemv_i8, which allocates its scratch per
call, on consecutive calls that reuse the library's fixed scratch array.  The
file is named so that pytest collects it last; it passes alone in a fresh
process and after the rest of the suite.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(lib, fn_name, x, w, ws, y, stream, *mem):
    import torch

    m, k = x.shape
    n = w.shape[0]
    return getattr(lib, fn_name)(x.data_ptr(), m, k, w.data_ptr(), ws.data_ptr(), n,
                                 y.data_ptr(), *mem, stream)


def test_gemv_noalloc_matches_allocating_entry_point(cuda):
    import torch

    from franken_ocr_b200._lib import MEM_DEVICE, check, lib

    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(2024)
    # two calls in a row with different shapes: the second reuses (and must
    # fully overwrite) the scratch the first one left behind
    for (m, k, n) in [(8, 1280, 1792), (3, 896, 1280)]:
        x = torch.randn((m, k), device="cuda", generator=g)
        w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda", generator=g)
        ws = torch.rand(n, device="cuda", generator=g) * 0.02 + 0.001
        y_ref = torch.empty((m, n), device="cuda")
        y_new = torch.full((m, n), float("nan"), device="cuda")
        check(_run(lib, "focr_gemv_i8", x, w, ws, y_ref, stream, MEM_DEVICE))
        check(_run(lib, "focr_gemv_i8_noalloc", x, w, ws, y_new, stream))
        torch.cuda.synchronize()
        # same kernels, same arithmetic: bit-identical (the tolerance the GEMV tests use)
        assert np.array_equal(y_new.cpu().numpy().view(np.uint32),
                              y_ref.cpu().numpy().view(np.uint32))


def test_gemv_noalloc_rejects_oversize(cuda):
    import torch

    from franken_ocr_b200._lib import FOCR_E_SHAPE, lib

    x = torch.zeros((300, 1280), device="cuda")   # 384000 bytes of activations > 262144
    w = torch.zeros((16, 1280), dtype=torch.int8, device="cuda")
    ws = torch.ones(16, device="cuda")
    y = torch.empty((300, 16), device="cuda")
    rc = _run(lib, "focr_gemv_i8_noalloc", x, w, ws, y, torch.cuda.current_stream().cuda_stream)
    assert rc == FOCR_E_SHAPE
    assert b"262144" in lib.focr_last_error()
