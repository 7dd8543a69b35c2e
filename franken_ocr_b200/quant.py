"""Offline weight quantisers (host, numpy): the formats the kernels consume.

* :func:`quantize_int8_f32` -- symmetric per-output-row int8
  (src/quant/int8.rs:110-163): ``scale = max|row| / 127`` (1.0 for an all-zero
  row), ``q = clamp(round_ties_even(w / scale), -127, 127)`` with TRUE division.
* :func:`pack_int4_f32` -- group int4 (src/quant/int4.rs:142-205):
  ``scale = max|group| / 7`` (1.0 if zero), ``q = clamp(ties_even(w / s), -8, 7)``,
  two nibbles per byte, low nibble = even column.

All arithmetic is float32 with IEEE rounding, so results are byte-identical to
the reference quantisers.
"""
from __future__ import annotations

import numpy as np


def _rowmax_abs(w: np.ndarray, axis: int) -> np.ndarray:
    # Rust's f32::max ignores NaN; np.fmax does the same.
    return np.fmax.reduce(np.abs(w), axis=axis, initial=np.float32(0.0)).astype(np.float32)


def quantize_int8_f32(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``[n, k]`` f32 -> (``[n, k]`` int8, ``[n]`` f32 scales)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("quantize_int8_f32: expected a 2-D [n, k] array")
    mx = _rowmax_abs(w, 1)
    zero = mx == np.float32(0.0)
    scale = np.where(zero, np.float32(1.0), mx / np.float32(127.0)).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        r = np.rint(w / scale[:, None])
    r = np.nan_to_num(r, nan=0.0, posinf=127.0, neginf=-127.0)
    q = np.clip(r, -127.0, 127.0).astype(np.int8)
    q[zero] = 0
    return q, scale


def pack_int4_f32(w: np.ndarray, group: int) -> tuple[np.ndarray, np.ndarray]:
    """``[n, k]`` f32 -> (``[n, k/2]`` packed u8, ``[n, k/group]`` f32 scales)."""
    if group not in (16, 32):
        raise ValueError(f"pack_int4_f32: group_size {group} must be 16 or 32")
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    if k % 2:
        raise ValueError(f"pack_int4_f32: k {k} must be even")
    if k % group:
        raise ValueError(f"pack_int4_f32: group_size {group} must divide k {k}")
    g = w.reshape(n, k // group, group)
    mx = _rowmax_abs(g, 2)
    scale = np.where(mx == np.float32(0.0), np.float32(1.0), mx / np.float32(7.0)).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        r = np.rint(g / scale[:, :, None])
    r = np.nan_to_num(r, nan=0.0, posinf=7.0, neginf=-8.0)
    q = np.clip(r, -8.0, 7.0).astype(np.int8).reshape(n, k)
    nib = (q.astype(np.uint8) & np.uint8(0x0F))
    packed = (nib[:, 0::2] | (nib[:, 1::2] << np.uint8(4))).astype(np.uint8)
    return np.ascontiguousarray(packed), np.ascontiguousarray(scale)


def unpack_int4(packed: np.ndarray, k: int) -> np.ndarray:
    """``[n, k/2]`` packed -> ``[n, k]`` int8 in [-8, 7] (simd/int4.rs:97-148)."""
    lo = (packed & 0x0F).astype(np.int8)
    hi = (packed >> 4).astype(np.int8)
    lo = np.where(lo >= 8, lo - 16, lo).astype(np.int8)
    hi = np.where(hi >= 8, hi - 16, hi).astype(np.int8)
    out = np.empty((packed.shape[0], k), dtype=np.int8)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    return out
