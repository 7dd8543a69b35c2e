"""Expert-parallel MoE layer and vocab-parallel lm-head over N GPUs.

Bindings of the library's multi-GPU entry points (``focr_comm_*``,
``focr_ep_*``, ``focr_top1_allgather``).  The data plane lives in the CUDA
library: dispatch writes each routed (token, slot) row -- int8 + scale, only
the routed ones -- into the owning rank's staging buffer over NVLink, the
owner's down GEMM writes each weighted partial back into the source rank's
return buffer, and the source sums them in slot order
(native_engine/decoder.rs:2231-2261), bit-identical to one GPU.  NCCL (loaded
by the library) bootstraps the peer mappings and carries the lm-head's
all-gather of per-shard top-1.

The reference is single-process; these classes have no counterpart there.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import MoeConfig, MoeWeights, check, lib
from .synth import MoeWeightsHost


def _stream():
    import torch

    return torch.cuda.current_stream().cuda_stream


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib.focr_nccl_unique_id(buf))
    return buf.raw


class Comm:
    """One rank of a communicator (collective create: every rank at once)."""

    def __init__(self, uid: bytes, rank: int, world: int):
        if len(uid) != 128:
            raise ValueError("the NCCL unique id is 128 bytes")
        self.rank, self.world = rank, world
        h = C.c_void_p()
        check(lib.focr_comm_create(C.c_char_p(uid), rank, world, C.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    def top1_allgather(self, best_val, best_idx):
        """Per-shard top-1 (device tensors [m]) -> (token u32 as int64 tensor,
        value) of the whole vocab on every rank."""
        import torch

        m = best_val.shape[0]
        tok = torch.empty(m, dtype=torch.int32, device=best_val.device)
        val = torch.empty(m, dtype=torch.float32, device=best_val.device)
        check(lib.focr_top1_allgather(self._h, best_val.data_ptr(), best_idx.data_ptr(), m,
                                      tok.data_ptr(), val.data_ptr(), _stream()))
        return tok.to(torch.int64) & 0xFFFFFFFF, val

    def close(self):
        if getattr(self, "_h", None):
            lib.focr_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()


def rank_weights(W: MoeWeightsHost, rank: int, world: int) -> MoeWeightsHost:
    """Rank's slice of W's routed experts + the router and the shared expert."""
    if W.n_experts % world:
        raise ValueError(f"{W.n_experts} experts do not split over {world} ranks")
    e = W.n_experts // world
    b = rank * e - W.expert_begin
    if b < 0 or b + e > W.expert_count:
        raise ValueError("weights do not hold this rank's experts")
    out = MoeWeightsHost(W.hidden, W.inter, W.n_experts, W.topk, W.shared_inter, rank * e, e,
                         W.group)
    out.router = W.router
    for k, v in W.arrays.items():
        out.arrays[k] = v if k.startswith("sh_") else np.ascontiguousarray(v[b:b + e])
    return out


class EpMoe:
    """Rank `rank` of an expert-parallel MoE layer (focr_ep_*).  ``W`` holds at
    least this rank's experts (a full layer is sliced)."""

    def __init__(self, W: MoeWeightsHost, rank: int, world: int, max_tokens: int,
                 norm_topk_prob: bool = True, routed_scaling_factor: float = 1.0):
        if W.expert_count != W.n_experts // world or W.expert_begin != rank * (W.n_experts // world):
            W = rank_weights(W, rank, world)
        self.rank, self.world, self.max_tokens = rank, world, max_tokens
        self.hidden, self.topk = W.hidden, W.topk
        cfg = MoeConfig(W.hidden, W.inter, W.n_experts, W.topk, W.shared_inter,
                        int(norm_topk_prob), float(routed_scaling_factor), W.group,
                        W.expert_begin, W.expert_count, max_tokens)
        wt = MoeWeights()
        keep = [np.ascontiguousarray(W.router, dtype=np.float32)]
        wt.router = keep[0].ctypes.data
        for name, arr in W.arrays.items():
            setattr(wt, name, arr.ctypes.data)
            keep.append(arr)
        h = C.c_void_p()
        check(lib.focr_ep_create(C.byref(cfg), C.byref(wt), rank, world, C.byref(h)))
        self._h = h
        del keep

    @property
    def handle(self):
        return self._h

    def ipc_handle(self) -> bytes:
        buf = C.create_string_buffer(64)
        check(lib.focr_ep_ipc_handle(self._h, buf))
        return buf.raw

    def connect(self, handles: list[bytes]):
        blob = b"".join(handles)
        check(lib.focr_ep_connect(self._h, C.c_char_p(blob)))

    def connect_comm(self, comm: Comm):
        check(lib.focr_ep_connect_comm(self._h, comm.handle))

    @staticmethod
    def connect_local(ranks: list["EpMoe"]):
        arr = (C.c_void_p * len(ranks))(*[r.handle.value for r in ranks])
        check(lib.focr_ep_connect_local(arr, len(ranks)))

    def forward(self, x, idx, w, y=None):
        import torch

        T = x.shape[0]
        y = torch.empty((T, self.hidden), dtype=torch.float32, device=x.device) if y is None else y
        check(lib.focr_ep_forward(self._h, x.data_ptr(), T, idx.data_ptr(), w.data_ptr(),
                                  y.data_ptr(), _stream()))
        return y

    def decode(self, x, y=None):
        import torch

        T = x.shape[0]
        y = torch.empty((T, self.hidden), dtype=torch.float32, device=x.device) if y is None else y
        idx = torch.empty((T, self.topk), dtype=torch.int32, device=x.device)
        w = torch.empty((T, self.topk), dtype=torch.float32, device=x.device)
        check(lib.focr_ep_decode(self._h, x.data_ptr(), T, y.data_ptr(), idx.data_ptr(),
                                 w.data_ptr(), _stream()))
        return y, idx, w

    def dispatch(self, x, idx, w):
        check(lib.focr_ep_dispatch(self._h, x.data_ptr(), x.shape[0], idx.data_ptr(),
                                   w.data_ptr(), _stream()))

    def experts(self):
        check(lib.focr_ep_experts(self._h, _stream()))

    def combine(self, y):
        check(lib.focr_ep_combine(self._h, y.data_ptr(), _stream()))
        return y

    def status(self) -> int:
        word = C.c_int(0)
        check(lib.focr_ep_status(self._h, C.byref(word)))
        return word.value

    def close(self):
        if getattr(self, "_h", None):
            lib.focr_ep_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()


def emulated_forward(ranks: list[EpMoe], xs, idxs, ws):
    """Run `len(ranks)` ranks that share one GPU, phase by phase on one stream
    (every wait is satisfied by an earlier launch): all dispatches, then all
    expert phases, then all combines."""
    import torch

    for r, x, i, w in zip(ranks, xs, idxs, ws):
        r.dispatch(x, i, w)
    for r in ranks:
        r.experts()
    return [r.combine(torch.empty((x.shape[0], r.hidden), dtype=torch.float32, device=x.device))
            for r, x in zip(ranks, xs)]
