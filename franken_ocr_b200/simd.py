"""Kernel tier: the B200 twin of franken_ocr's ``src/simd`` public API.

Same names, argument meaning and error behaviour as the reference:

* ``igemm_s8s8(a, b, m, k, n, out)`` -- ``out[M,N] += a[M,K] . b[N,K]^T`` in
  int32 (src/simd/dispatch.rs:246).
* ``igemm_u8s8(a, b, m, k, n, out)`` -- unsigned activations
  (src/simd/dispatch.rs:276).
* ``igemm_s4s8_packed(a, b_packed, scales, group, m, k, n, out)`` -- packed
  int4 weights, f32 out overwritten (src/simd/int4.rs:437).
* ``tier_string()`` / ``selftest()`` (src/simd/dispatch.rs:128-136, :376).

Arrays are either host numpy arrays (copied to the GPU and back) or CUDA
torch tensors (device pointers, enqueued on torch's current stream).  A
contract violation raises :class:`FocrError` carrying the reference's panic
text (e.g. ``"igemm_s8s8: a.len 2 != m*k 1"``).
"""
from __future__ import annotations

import ctypes as C
import json

import numpy as np

from ._lib import MEM_DEVICE, MEM_HOST, FocrError, check, lib

__all__ = [
    "FocrError", "igemm_s8s8", "igemm_u8s8", "igemm_s4s8_packed", "quantize_rows_i8",
    "gemv_i8", "tier_string", "selftest",
]


def _is_torch_cuda(x) -> bool:
    return type(x).__module__.startswith("torch") and getattr(x, "is_cuda", False)


def _arg(x, np_dtype, name: str):
    """(pointer, element count, mem kind) for a numpy array or CUDA tensor."""
    if _is_torch_cuda(x):
        if not x.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        return x.data_ptr(), x.numel(), MEM_DEVICE
    arr = x
    if not isinstance(arr, np.ndarray):
        raise TypeError(f"{name}: expected numpy array or CUDA tensor, got {type(x).__name__}")
    if arr.dtype != np_dtype:
        raise TypeError(f"{name}: dtype {arr.dtype} != {np.dtype(np_dtype)}")
    if not arr.flags.c_contiguous:
        raise ValueError(f"{name} must be C-contiguous")
    return arr.ctypes.data, arr.size, MEM_HOST


def _stream(mem: int):
    if mem == MEM_DEVICE:
        import torch

        return torch.cuda.current_stream().cuda_stream
    return None


def _mem_of(args):
    kinds = {a[2] for a in args}
    if len(kinds) != 1:
        raise ValueError("mix of host arrays and device tensors")
    return kinds.pop()


def igemm_s8s8(a, b, m: int, k: int, n: int, out) -> None:
    """``out[M,N] += a[M,K] (i8) . b[N,K] (i8, output-channel-major)^T``."""
    pa, pb, po = _arg(a, np.int8, "a"), _arg(b, np.int8, "b"), _arg(out, np.int32, "out")
    mem = _mem_of((pa, pb, po))
    check(lib.focr_igemm_s8s8(pa[0], pa[1], pb[0], pb[1], m, k, n, po[0], po[1], mem, _stream(mem)))


def igemm_u8s8(a, b, m: int, k: int, n: int, out) -> None:
    """``out[M,N] += a[M,K] (u8) . b[N,K] (i8)^T``."""
    pa, pb, po = _arg(a, np.uint8, "a"), _arg(b, np.int8, "b"), _arg(out, np.int32, "out")
    mem = _mem_of((pa, pb, po))
    check(lib.focr_igemm_u8s8(pa[0], pa[1], pb[0], pb[1], m, k, n, po[0], po[1], mem, _stream(mem)))


def igemm_s4s8_packed(a, b_packed, scales, group: int, m: int, k: int, n: int, out) -> None:
    """``out[m,n] = sum_g scales[n,g] * f32(dot over group g)`` (overwrite)."""
    pa = _arg(a, np.int8, "a")
    pb = _arg(b_packed, np.uint8, "b_packed")
    ps = _arg(scales, np.float32, "scales")
    po = _arg(out, np.float32, "out")
    mem = _mem_of((pa, pb, ps, po))
    check(lib.focr_igemm_s4s8_packed(pa[0], pa[1], pb[0], pb[1], ps[0], ps[1], group, m, k, n,
                                     po[0], po[1], mem, _stream(mem)))


def quantize_rows_i8(x, m: int, k: int, xq, scales, ties_even: bool = False) -> None:
    """Per-row dynamic int8 quantisation (decoder.rs:1588-1597 / :1647-1656)."""
    px, pq, ps = _arg(x, np.float32, "x"), _arg(xq, np.int8, "xq"), _arg(scales, np.float32, "scales")
    mem = _mem_of((px, pq, ps))
    if px[1] != m * k or pq[1] != m * k or ps[1] != m:
        raise FocrError(-1, "quantize_rows_i8: length mismatch")
    check(lib.focr_quantize_rows_i8(px[0], m, k, int(ties_even), pq[0], ps[0], mem, _stream(mem)))


def gemv_i8(x, m: int, k: int, w, w_scale, n: int, y) -> None:
    """``y = ((f32)(Q(x) . w^T) * a_scale) * w_scale`` (decoder.rs:1607)."""
    px, pw, ps, py = (_arg(x, np.float32, "x"), _arg(w, np.int8, "w"),
                      _arg(w_scale, np.float32, "w_scale"), _arg(y, np.float32, "y"))
    mem = _mem_of((px, pw, ps, py))
    if px[1] != m * k or pw[1] != n * k or ps[1] != n or py[1] != m * n:
        raise FocrError(-1, "gemv_i8: length mismatch")
    check(lib.focr_gemv_i8(px[0], m, k, pw[0], ps[0], n, py[0], mem, _stream(mem)))


def tier_string() -> str:
    """The dispatched tier (``"sm100a"``), as ``robot backends`` reports it."""
    return lib.focr_tier_string().decode()


def selftest() -> dict:
    """Run the reference's selftest battery on the GPU tier; returns the report."""
    buf = C.create_string_buffer(1 << 16)
    ok = C.c_int(0)
    check(lib.focr_selftest(buf, len(buf), C.byref(ok)))
    rep = json.loads(buf.value.decode())
    rep["all_ok"] = bool(ok.value)
    return rep
