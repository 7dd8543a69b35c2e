"""Decoder pieces beside the MoE layer (the config-3 decoder), mirroring the
reference's functions:

* ``rms_norm(x, weight, eps)`` -- ``nn::rms_norm`` (native_engine/nn.rs:240);
* ``apply_rope(x, cos, sin, head_dim)`` -- ``apply_rope``
  (native_engine/decoder.rs:229), in place, with a ``RopeTable``
  (decoder.rs:171) built on the host as the reference does;
* ``attention_decode(q, ref_k, ref_v, prefill_len, ring_k, ring_v, ring_len)``
  -- ``rswa::decode_attention`` (native_engine/rswa.rs:855) over head-major
  ``[heads][stride][head_dim]`` caches.

Arguments are numpy arrays (host) or CUDA tensors (device), not mixed.
"""
from __future__ import annotations

import numpy as np

from ._lib import check, lib
from .simd import _arg, _mem_of, _stream


def rms_norm(x, weight=None, eps: float = 1e-6, y=None):
    rows, cols = x.shape
    if y is None:
        y = np.empty_like(x) if isinstance(x, np.ndarray) else x.new_empty(x.shape)
    args = [_arg(x, np.float32, "x"), _arg(y, np.float32, "y")]
    pw = _arg(weight, np.float32, "weight") if weight is not None else None
    if pw is not None:
        args.append(pw)
        if pw[1] != cols:
            raise ValueError(f"rms_norm: weight len {pw[1]} != cols {cols}")
    mem = _mem_of(args)
    check(lib.focr_rms_norm(args[0][0], rows, cols, pw[0] if pw else None, float(eps), args[1][0],
                            mem, _stream(mem)))
    return y


def apply_rope(x, cos_t, sin_t, head_dim: int):
    seq, cols = x.shape
    args = [_arg(x, np.float32, "x"), _arg(cos_t, np.float32, "cos"), _arg(sin_t, np.float32, "sin")]
    mem = _mem_of(args)
    check(lib.focr_rope_apply(args[0][0], seq, cols, head_dim, args[1][0], args[2][0], mem,
                              _stream(mem)))
    return x


def attention_decode(q, ref_k, ref_v, prefill_len: int, ring_k, ring_v, ring_len: int, out=None):
    """q [heads, head_dim]; caches [heads, stride, head_dim] (row r of head h)."""
    heads, head_dim = q.shape
    if out is None:
        out = np.empty_like(q) if isinstance(q, np.ndarray) else q.new_empty(q.shape)
    args = [_arg(q, np.float32, "q"), _arg(out, np.float32, "out"),
            _arg(ref_k, np.float32, "ref_k"), _arg(ref_v, np.float32, "ref_v"),
            _arg(ring_k, np.float32, "ring_k"), _arg(ring_v, np.float32, "ring_v")]
    mem = _mem_of(args)
    check(lib.focr_attention_decode(args[0][0], args[2][0], args[3][0], prefill_len,
                                    ref_k.shape[1], args[4][0], args[5][0], ring_len,
                                    ring_k.shape[1], heads, head_dim, args[1][0], mem,
                                    _stream(mem)))
    return out
