"""Expert-parallel MoE layer over N GPUs (one process per GPU).

The reference has no distributed code (it runs the 6 routed experts of a
token as rayon tasks, native_engine/decoder.rs:2231-2252); this module splits
the same computation by expert: rank r owns routed experts
[r*E/N, (r+1)*E/N) and a replica of the fused shared expert.  One forward of
T local tokens with given routing (idx, w of shape [T, topk]):

1. dispatch -- focr_ep_pack places every (token, slot) pair in the block of
   rows reserved for the rank owning its expert (fixed capacity C =
   max_tokens*topk rows per peer, unused rows marked with expert id -1): the
   token's f32 row plus (global expert id, routing weight).  Two equal-split
   all-to-alls move the blocks; no host synchronisation is needed.  The
   receiver quantises the rows itself, which reproduces the sender's
   quantisation exactly (row quantisation is deterministic).
2. experts -- one focr_moe_forward_rows call on the rank's layer (its expert
   subset + the shared expert) over [N*C received pairs | T own tokens]: each
   received pair is a one-slot row whose output is p = expert(x) * w,
   bit-identical to the partial the single-GPU layer forms
   (decoder.rs:2236-2247); the own tokens (ids -1) get the shared expert.
3. return -- the partials travel back by the reverse all-to-all and
   focr_moe_combine gathers them per (token, slot) and forms
   ((0 + p_0) + ... + p_{k-1}) + s (decoder.rs:2253-2261).
"""
from __future__ import annotations

import numpy as np

from ._lib import check, lib
from .moe import MoeLayer
from .synth import MoeWeightsHost


def rank_weights(W: MoeWeightsHost, rank: int, world: int) -> MoeWeightsHost:
    """Rank's slice of W's routed experts + W's shared expert, as a one-slot
    layer (each received pair is a row with one routed expert)."""
    if W.n_experts % world:
        raise ValueError(f"{W.n_experts} experts do not split over {world} ranks")
    e = W.n_experts // world
    b = rank * e - W.expert_begin
    if b < 0 or b + e > W.expert_count:
        raise ValueError("weights do not hold this rank's experts")
    out = MoeWeightsHost(W.hidden, W.inter, W.n_experts, 1, W.shared_inter, rank * e, e, W.group)
    out.router = W.router
    for k, v in W.arrays.items():
        out.arrays[k] = v if k.startswith("sh_") else np.ascontiguousarray(v[b:b + e])
    return out


class EpMoeRank:
    """One rank of an expert-parallel MoE layer (device tensors, torch)."""

    def __init__(self, W: MoeWeightsHost, rank: int, world: int, max_tokens: int):
        import torch

        self.rank, self.world = rank, world
        self.hidden, self.topk = W.hidden, W.topk
        self.e_local = W.n_experts // world
        self.max_tokens = max_tokens
        self.cap = max_tokens * W.topk        # rows reserved per peer
        self.layer = MoeLayer(rank_weights(W, rank, world),
                              max_tokens=world * self.cap + max_tokens)
        dev = torch.device("cuda", torch.cuda.current_device())
        n = world * self.cap
        self.send_x = torch.empty((n, self.hidden), dtype=torch.float32, device=dev)
        self.send_meta = torch.empty((n, 2), dtype=torch.int32, device=dev)
        self.recv_x = torch.empty((n + max_tokens, self.hidden), dtype=torch.float32, device=dev)
        self.recv_meta = torch.empty((n + max_tokens, 2), dtype=torch.int32, device=dev)
        self.rows = torch.empty(max_tokens * self.topk, dtype=torch.int32, device=dev)
        self.out = torch.empty((n + max_tokens, self.hidden), dtype=torch.float32, device=dev)
        self.back = torch.empty((n, self.hidden), dtype=torch.float32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)

    def _stream(self):
        import torch

        return torch.cuda.current_stream().cuda_stream

    def pack(self, x, idx, w):
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > max_tokens {self.max_tokens}")
        check(lib.focr_ep_pack(x.data_ptr(), idx.data_ptr(), w.data_ptr(), T, self.topk,
                               self.hidden, self.e_local, self.world, self.cap,
                               self.send_x.data_ptr(), self.send_meta.data_ptr(),
                               self.recv_x.data_ptr(), self.recv_meta.data_ptr(),
                               self.rows.data_ptr(), self.status.data_ptr(), self._stream()))

    def experts(self, T):
        """Forward over [received pairs | own tokens] (recv buffers filled)."""
        import torch

        n = self.world * self.cap
        m = n + T
        ridx = self.recv_meta[:m, 0:1].contiguous()
        rw = self.recv_meta[:m, 1:2].contiguous().view(torch.float32)
        return self.layer.forward_rows(self.recv_x[:m], ridx, rw, n, self.out[:m])

    def combine(self, T, back):
        import torch

        n = self.world * self.cap
        y = torch.empty((T, self.hidden), dtype=torch.float32, device=back.device)
        check(lib.focr_moe_combine(back.data_ptr(), self.rows.data_ptr(),
                                   self.out[n:].data_ptr(), T, self.topk, self.hidden,
                                   y.data_ptr(), self._stream()))
        return y

    def forward(self, x, idx, w, group=None):
        """Distributed forward over torch.distributed (NCCL) for this rank."""
        import torch.distributed as dist

        T = x.shape[0]
        n = self.world * self.cap
        self.pack(x, idx, w)
        if self.world == 1:
            self.recv_x[:n].copy_(self.send_x)
            self.recv_meta[:n].copy_(self.send_meta)
        else:
            dist.all_to_all_single(self.recv_x[:n], self.send_x, group=group)
            dist.all_to_all_single(self.recv_meta[:n], self.send_meta, group=group)
        self.experts(T)
        if self.world == 1:
            back = self.out[:n]
        else:
            dist.all_to_all_single(self.back, self.out[:n], group=group)
            back = self.back
        return self.combine(T, back)

    def close(self):
        self.layer.close()


def emulated_forward(ranks, xs, idxs, ws):
    """Run the expert-parallel forward of len(ranks) ranks on one device,
    doing the equal-split all-to-alls by slicing (the exchange under test)."""
    import torch

    N = len(ranks)
    C = ranks[0].cap
    for r, x, i, w in zip(ranks, xs, idxs, ws):
        r.pack(x, i, w)
    for d in range(N):
        ranks[d].recv_x[:N * C] = torch.cat([ranks[s].send_x[d * C:(d + 1) * C] for s in range(N)])
        ranks[d].recv_meta[:N * C] = torch.cat([ranks[s].send_meta[d * C:(d + 1) * C]
                                                for s in range(N)])
    for d in range(N):
        ranks[d].experts(xs[d].shape[0])
    ys = []
    for s in range(N):
        back = torch.cat([ranks[d].out[s * C:(s + 1) * C] for d in range(N)])
        ys.append(ranks[s].combine(xs[s].shape[0], back))
    return ys
