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
    # calls in a row with different shapes: each reuses (and must fully
    # overwrite) the scratch the previous one left behind.  m = 1 is the decode
    # row (the fused in-kernel-quantising GEMV on both entry points), m = 9
    # spans two eight-row GEMV chunks, m = 1024 fills the scratch exactly.
    for (m, k, n) in [(8, 1280, 1792), (3, 896, 1280), (1, 1280, 1792), (9, 896, 1280),
                      (1024, 256, 64), (2, 1280, 1792)]:
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
    # one row within the scratch but wider than the GEMV's shared-memory stage
    x1 = torch.zeros((1, 262144), device="cuda")
    w1 = torch.zeros((4, 262144), dtype=torch.int8, device="cuda")
    y1 = torch.empty((1, 4), device="cuda")
    rc = _run(lib, "focr_gemv_i8_noalloc", x1, w1, torch.ones(4, device="cuda"), y1,
              torch.cuda.current_stream().cuda_stream)
    assert rc == FOCR_E_SHAPE
    assert b"204800" in lib.focr_last_error()
