"""Vocab-sharded int8 lm-head with greedy top-1 (decoder.rs:2275-2296 lm head,
decoder.rs:1851-1927 vocab tiles, sampler.rs:168-186 argmax_row)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import MEM_DEVICE, MEM_HOST, check, lib


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()


class LmHeadShard:
    """Rows [row_begin, row_begin + rows) of the [vocab, hidden] int8 head, or
    of an int4 head (``group`` 16/32: ``w`` packed [rows, hidden/2],
    ``scales`` [rows, hidden/group])."""

    def __init__(self, w: np.ndarray, scales: np.ndarray, row_begin: int = 0, max_tokens: int = 1,
                 group: int = 0):
        scales = np.ascontiguousarray(scales, dtype=np.float32)
        self.row_begin = row_begin
        h = C.c_void_p()
        if group:
            w = np.ascontiguousarray(w, dtype=np.uint8)
            self.rows, self.hidden = w.shape[0], w.shape[1] * 2
            check(lib.focr_lmhead_create_s4(w.ctypes.data, scales.ctypes.data, group, self.rows,
                                            self.hidden, row_begin, max_tokens, C.byref(h)))
        else:
            w = np.ascontiguousarray(w, dtype=np.int8)
            self.rows, self.hidden = w.shape
            check(lib.focr_lmhead_create(w.ctypes.data, scales.ctypes.data, self.rows, self.hidden,
                                         row_begin, max_tokens, C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib.focr_lmhead_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def top1(self, x, want_logits: bool = False):
        """Per row: (best value, best GLOBAL index or -1, shard logits or None)."""
        m = x.shape[0]
        if isinstance(x, np.ndarray):
            x = np.ascontiguousarray(x, dtype=np.float32)
            bv = np.empty(m, np.float32)
            bi = np.empty(m, np.int32)
            lg = np.empty((m, self.rows), np.float32) if want_logits else None
            check(lib.focr_lmhead_top1(self._h, x.ctypes.data, m, bv.ctypes.data, bi.ctypes.data,
                                       _ptr(lg), MEM_HOST, None))
            return bv, bi, lg
        import torch

        bv = torch.empty(m, dtype=torch.float32, device=x.device)
        bi = torch.empty(m, dtype=torch.int32, device=x.device)
        lg = torch.empty((m, self.rows), dtype=torch.float32, device=x.device) if want_logits else None
        check(lib.focr_lmhead_top1(self._h, x.data_ptr(), m, bv.data_ptr(), bi.data_ptr(),
                                   _ptr(lg), MEM_DEVICE, torch.cuda.current_stream().cuda_stream))
        return bv, bi, lg


def top1_combine(vals: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """[shards, m] per-shard (value, global index) -> argmax_row token per row."""
    vals = np.ascontiguousarray(vals, dtype=np.float32)
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    shards, m = vals.shape
    tok = np.empty(m, dtype=np.uint32)
    check(lib.focr_top1_combine(vals.ctypes.data, idx.ctypes.data, shards, m, tok.ctypes.data))
    return tok
