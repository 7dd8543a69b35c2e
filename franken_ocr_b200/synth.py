"""Seeded synthetic inputs for the benchmark configurations.

There is no model checkpoint or dataset here: weights are drawn N(0, 0.02)
(router f32, experts quantised per row to int8, or group-int4) and hidden
states N(0, 1), each array from its own numpy PCG64 stream keyed by
(seed, role, expert) so that an expert-parallel rank can draw exactly the
experts it owns.  Routing for the batched configuration is drawn so that
expert loads follow a Zipf(1.1) skew over the experts, six distinct experts
per token.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .quant import pack_int4_f32, quantize_int8_f32

HIDDEN = 1280
INTER = 896
N_EXPERTS = 64
TOPK = 6
SHARED_INTER = 1792
VOCAB = 129280
WEIGHT_STD = 0.02

_ROLE = {"router": 1, "gate": 2, "up": 3, "down": 4, "sh_gate": 5, "sh_up": 6, "sh_down": 7,
         "x": 8, "route": 9, "lm_head": 10, "q": 11, "k": 12, "v": 13, "o": 14,
         "dense_gate": 15, "dense_up": 16, "dense_down": 17, "norm": 18, "embed": 19,
         "prompt": 20}


def rng(seed: int, role: str, idx: int = 0) -> np.random.Generator:
    return np.random.default_rng([int(seed), _ROLE[role], int(idx)])


def normal(seed: int, role: str, idx: int, shape, std: float) -> np.ndarray:
    return (rng(seed, role, idx).standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(
        np.float32)


def _parallel(fn, n: int) -> None:
    """fn(0..n-1) on a thread pool: numpy's generators and ufuncs release the
    GIL on large arrays, and every index draws from its own stream, so the
    result does not depend on scheduling."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    workers = min(n, os.cpu_count() or 1, 32)
    if workers <= 1:
        for i in range(n):
            fn(i)
        return
    with ThreadPoolExecutor(workers) as ex:
        list(ex.map(fn, range(n)))


@dataclass
class MoeWeightsHost:
    hidden: int
    inter: int
    n_experts: int
    topk: int
    shared_inter: int
    expert_begin: int
    expert_count: int
    group: int = 0
    router: np.ndarray = None
    arrays: dict = field(default_factory=dict)


def moe_layer(seed: int, hidden: int = HIDDEN, inter: int = INTER, n_experts: int = N_EXPERTS,
              topk: int = TOPK, shared_inter: int = 0, expert_begin: int = 0,
              expert_count: int | None = None, group: int = 0) -> MoeWeightsHost:
    """Weights of one MoE layer (experts [expert_begin, expert_begin+count))."""
    if expert_count is None:
        expert_count = n_experts - expert_begin
    W = MoeWeightsHost(hidden, inter, n_experts, topk, shared_inter, expert_begin, expert_count,
                       group)
    W.router = normal(seed, "router", 0, (n_experts, hidden), WEIGHT_STD)
    E = expert_count
    shapes = {"gate": (inter, hidden), "up": (inter, hidden), "down": (hidden, inter)}
    for role, shp in shapes.items():
        if group:
            qs = [pack_int4_f32(normal(seed, role, expert_begin + e, shp, WEIGHT_STD), group)
                  for e in range(E)]
            W.arrays[role + "_p"] = np.ascontiguousarray(np.stack([q for q, _ in qs]))
            W.arrays[role + "_gs"] = np.ascontiguousarray(np.stack([s for _, s in qs]))
        else:
            q = np.empty((E,) + shp, dtype=np.int8)
            s = np.empty((E, shp[0]), dtype=np.float32)

            def one(e, role=role, shp=shp, q=q, s=s):
                q[e], s[e] = quantize_int8_f32(normal(seed, role, expert_begin + e, shp, WEIGHT_STD))

            _parallel(one, E)
            W.arrays[role + "_w"] = q
            W.arrays[role + "_s"] = s
    if shared_inter:
        for role, shp in (("sh_gate", (shared_inter, hidden)), ("sh_up", (shared_inter, hidden)),
                          ("sh_down", (hidden, shared_inter))):
            q, s = quantize_int8_f32(normal(seed, role, 0, shp, WEIGHT_STD))
            W.arrays[role + "_w"] = q
            W.arrays[role + "_s"] = s
    return W


def hidden_states(seed: int, m: int, hidden: int = HIDDEN, idx: int = 0) -> np.ndarray:
    return normal(seed, "x", idx, (m, hidden), 1.0)


def zipf_routing(seed: int, m: int, n_experts: int = N_EXPERTS, topk: int = TOPK,
                 s: float = 1.1, idx: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Top-k routing with Zipf(s) expert popularity: for each token, ``topk``
    distinct experts drawn without replacement with P(e) ~ 1/(rank+1)^s over a
    seeded random rank order; weights are a softmax of N(0,1) scores sorted
    descending (the router's output order) and renormalised."""
    g = rng(seed, "route", idx)
    rank = g.permutation(n_experts)
    p = 1.0 / np.power(np.arange(1, n_experts + 1, dtype=np.float64), s)
    p = p / p.sum()
    prob = p[rank]  # expert e has popularity p[rank[e]]
    idx_out = np.empty((m, topk), dtype=np.int32)
    w_out = np.empty((m, topk), dtype=np.float32)
    for t in range(m):
        chosen = g.choice(n_experts, size=topk, replace=False, p=prob)
        sc = np.sort(g.standard_normal(topk))[::-1]
        e = np.exp(sc - sc.max())
        wv = (e / e.sum()).astype(np.float32)
        idx_out[t] = chosen
        w_out[t] = wv
    return idx_out, w_out


def lm_head(seed: int, rows: int, hidden: int = HIDDEN, row_begin: int = 0,
            block: int = 16160) -> tuple[np.ndarray, np.ndarray]:
    """Rows [row_begin, row_begin+rows) of an int8 [VOCAB, hidden] head, drawn
    in fixed blocks so any shard reproduces the monolithic head."""
    q = np.empty((rows, hidden), dtype=np.int8)
    s = np.empty(rows, dtype=np.float32)
    r = row_begin
    while r < row_begin + rows:
        b = r // block
        b0, b1 = b * block, (b + 1) * block
        full = normal(seed, "lm_head", b, (block, hidden), WEIGHT_STD)
        lo, hi = max(r, b0), min(row_begin + rows, b1)
        qq, ss = quantize_int8_f32(full[lo - b0:hi - b0])
        q[lo - row_begin:hi - row_begin] = qq
        s[lo - row_begin:hi - row_begin] = ss
        r = hi
    return q, s


DENSE_INTER = 6848
N_LAYERS = 12
HEADS = 10


def decoder_model(seed: int, layers: int = N_LAYERS, hidden: int = HIDDEN, heads: int = HEADS,
                  n_experts: int = N_EXPERTS, topk: int = TOPK, inter: int = INTER,
                  shared_inter: int = SHARED_INTER, dense_inter: int = DENSE_INTER,
                  vocab: int = VOCAB, first_dense: int = 1):
    """A synthetic int8 decoder with the reference's layout (decoder.rs:2001-2117):
    layers ``[0, first_dense)`` dense SwiGLU, the rest MoE (``n_experts``
    routed top-``topk`` plus one shared expert of ``shared_inter`` = the two
    shared experts of 896 fused), heads x 128 attention, RMSNorm weights
    1 + N(0, 0.05), projections N(0, 0.02) quantised per row, f32 embeddings
    N(0, 1).  Layer ``l``'s arrays are drawn from seed ``seed * 1000 + l``."""
    from .decoder import HEAD_DIM, DecoderWeightsHost, LayerWeightsHost

    D = heads * HEAD_DIM
    Ls = []
    for li in range(layers):
        ls = seed * 1000 + li
        L = LayerWeightsHost(
            input_ln=(1.0 + normal(ls, "norm", 0, (hidden,), 0.05)).astype(np.float32),
            post_ln=(1.0 + normal(ls, "norm", 1, (hidden,), 0.05)).astype(np.float32))
        for r, shp in (("q", (D, hidden)), ("k", (D, hidden)), ("v", (D, hidden)),
                       ("o", (hidden, D))):
            L.proj[r + "_w"], L.proj[r + "_s"] = quantize_int8_f32(normal(ls, r, 0, shp, WEIGHT_STD))
        if li < first_dense:
            L.dense = {}
            for r, shp in (("gate", (dense_inter, hidden)), ("up", (dense_inter, hidden)),
                           ("down", (hidden, dense_inter))):
                L.dense[r + "_w"], L.dense[r + "_s"] = quantize_int8_f32(
                    normal(ls, "dense_" + r, 0, shp, WEIGHT_STD))
        else:
            L.moe = moe_layer(ls, hidden=hidden, inter=inter, n_experts=n_experts, topk=topk,
                              shared_inter=shared_inter)
        Ls.append(L)
    lm_w, lm_s = lm_head(seed, vocab, hidden=hidden, block=min(16160, vocab))
    return DecoderWeightsHost(
        hidden=hidden, heads=heads, vocab=vocab, layers=Ls,
        final_norm=(1.0 + normal(seed, "norm", 2, (hidden,), 0.05)).astype(np.float32),
        lm_w=lm_w, lm_s=lm_s, embed=normal(seed, "embed", 0, (vocab, hidden), 1.0))


def prompt_embeds(seed: int, seq: int, hidden: int = HIDDEN) -> np.ndarray:
    """Prefill input embeddings N(0, 1) ``[seq, hidden]``."""
    return normal(seed, "prompt", 0, (seq, hidden), 1.0)
