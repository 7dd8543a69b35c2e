"""MoE decode layer on the GPU: the device twin of the int8 engine's MoE arm.

``MoeLayer`` uploads one layer's weights once (DecoderWeightCacheI8::build,
native_engine/decoder.rs:2018) and exposes

* :meth:`route` -- ``moe::route`` (native_engine/moe.rs:181-266),
* :meth:`forward` -- expert FFN + combine for a given routing,
* :meth:`decode` -- route + forward (``decode_mlp_i8``, decoder.rs:2199-2268;
  for m > 1 the per-stream batched semantics of decoder.rs:2812-2933).

Inputs/outputs are host numpy arrays or CUDA torch tensors (device mode,
enqueued on torch's current stream).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import MEM_DEVICE, MEM_HOST, MoeConfig, MoeWeights, check, lib
from .synth import MoeWeightsHost


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        if not a.flags.c_contiguous:
            raise ValueError("array must be C-contiguous")
        return a.ctypes.data
    return a.data_ptr()


def _mem(x):
    return MEM_HOST if isinstance(x, np.ndarray) else MEM_DEVICE


def _stream(mem):
    if mem == MEM_DEVICE:
        import torch

        return torch.cuda.current_stream().cuda_stream
    return None


class MoeLayer:
    def __init__(self, W: MoeWeightsHost, max_tokens: int = 1, norm_topk_prob: bool = True,
                 routed_scaling_factor: float = 1.0):
        self.hidden, self.topk = W.hidden, W.topk
        self.n_experts = W.n_experts
        self.expert_begin, self.expert_count = W.expert_begin, W.expert_count
        self.max_tokens = max_tokens
        cfg = MoeConfig(W.hidden, W.inter, W.n_experts, W.topk, W.shared_inter,
                        int(norm_topk_prob), float(routed_scaling_factor), W.group,
                        W.expert_begin, W.expert_count, max_tokens)
        wt = MoeWeights()
        wt.router = _ptr(np.ascontiguousarray(W.router, dtype=np.float32))
        keep = [W.router]
        for name, arr in W.arrays.items():
            setattr(wt, name, _ptr(arr))
            keep.append(arr)
        h = C.c_void_p()
        check(lib.focr_moe_create(C.byref(cfg), C.byref(wt), C.byref(h)))
        self._h = h
        del keep

    def close(self):
        if getattr(self, "_h", None):
            lib.focr_moe_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def _out(self, like, shape, dtype):
        if isinstance(like, np.ndarray):
            return np.empty(shape, dtype=dtype)
        import torch

        tdt = {np.float32: torch.float32, np.int32: torch.int32}[dtype]
        return torch.empty(shape, dtype=tdt, device=like.device)

    def route(self, x, idx=None, w=None):
        m = x.shape[0]
        idx = self._out(x, (m, self.topk), np.int32) if idx is None else idx
        w = self._out(x, (m, self.topk), np.float32) if w is None else w
        mem = _mem(x)
        check(lib.focr_moe_route(self._h, _ptr(x), m, _ptr(idx), _ptr(w), mem, _stream(mem)))
        return idx, w

    def forward(self, x, idx, w, y=None):
        m = x.shape[0]
        y = self._out(x, (m, self.hidden), np.float32) if y is None else y
        mem = _mem(x)
        check(lib.focr_moe_forward(self._h, _ptr(x), m, _ptr(idx), _ptr(w), _ptr(y), mem,
                                   _stream(mem)))
        return y

    def forward_rows(self, x, idx, w, shared_begin, y=None):
        """forward with the shared expert on rows >= shared_begin only; ids < 0
        are empty slots (device tensors)."""
        import torch

        m = x.shape[0]
        y = torch.empty((m, self.hidden), dtype=torch.float32, device=x.device) if y is None else y
        check(lib.focr_moe_forward_rows(self._h, x.data_ptr(), m, idx.data_ptr(), w.data_ptr(),
                                        y.data_ptr(), shared_begin,
                                        torch.cuda.current_stream().cuda_stream))
        return y

    def decode(self, x, y=None, idx=None, w=None):
        m = x.shape[0]
        y = self._out(x, (m, self.hidden), np.float32) if y is None else y
        idx = self._out(x, (m, self.topk), np.int32) if idx is None else idx
        w = self._out(x, (m, self.topk), np.float32) if w is None else w
        mem = _mem(x)
        check(lib.focr_moe_decode(self._h, _ptr(x), m, _ptr(y), _ptr(idx), _ptr(w), mem,
                                  _stream(mem)))
        return y, idx, w

    def prefill(self, x, y=None, idx=None, w=None):
        """moe_block_i8 (decoder.rs:2142-2181): ties-even activation
        quantisation, partials summed in ascending expert order."""
        m = x.shape[0]
        y = self._out(x, (m, self.hidden), np.float32) if y is None else y
        idx = self._out(x, (m, self.topk), np.int32) if idx is None else idx
        w = self._out(x, (m, self.topk), np.float32) if w is None else w
        mem = _mem(x)
        check(lib.focr_moe_prefill(self._h, _ptr(x), m, _ptr(y), _ptr(idx), _ptr(w), mem,
                                   _stream(mem)))
        return y, idx, w
