"""The int8 decoder on the GPU: prefill, R-SWA decode steps and greedy decode.

Mirrors the reference's int8 decode engine:

* :class:`DecoderWeightsHost` -- ``DecoderWeightCacheI8`` (decoder.rs:2001-2117):
  per layer the two RMSNorm weights, int8 q/k/v/o projections, and either
  the dense SwiGLU MLP (layer 0) or a MoE layer; the final norm, the int8
  lm-head and the f32 token-embedding table;
* :meth:`DecoderI8.prefill` -- ``prefill_with_cache_i8`` (decoder.rs:2412-2540,
  monolithic schedule): ties-even int8 projections, RoPE at positions
  ``0..seq``, causal attention, MoE prefill, and the prefill K/V recorded as
  each layer's permanent reference block (``RingCache::record_prefill``,
  rswa.rs:389);
* :meth:`DecoderI8.decode_step` -- ``decode_step_with_cache_i8``
  (decoder.rs:2542-2640): half-away int8 GEMVs (q/k/v as one fused GEMV,
  byte-identical per row), RoPE at the true position, the ring write
  (``write_decode_step``, rswa.rs:451-500: append until 128 rows, then
  overwrite the oldest slot) and decode attention over reference ++ ring;
* :meth:`DecoderI8.lm_head_top1` -- ``lm_head_cached_i8`` (decoder.rs:2275)
  + ``sampler::argmax_row`` (sampler.rs:168);
* :meth:`DecoderI8.generate` -- the greedy loop of ``generate_cached_i8``
  (native_engine/mod.rs:1860-1898): token ``i`` is decoded at position
  ``prefill_len + i - 1``.  There is no EOS stop: a fixed number of tokens is
  produced, as the benchmark configuration asks.

Every op is a call into ``libfocr_cuda.so`` on torch's current stream; torch
only allocates device memory and copies rows (embedding lookup, ring writes,
reference-block layout).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

import ctypes as C

from ._lib import (MEM_DEVICE, MEM_HOST, DecoderConfig, DecoderLayerWeights, DecoderWeights,
                   MoeConfig, MoeWeights, check, lib)
from .synth import MoeWeightsHost

HEAD_DIM = 128
RING_WINDOW = 128
ROPE_THETA = 10000.0
RMS_NORM_EPS = 1e-6


@dataclass
class LayerWeightsHost:
    """One decoder layer: norms f32 ``[hidden]``; projections int8 ``[out, in]``
    with per-row f32 scales; ``dense`` = dict of gate/up/down ``_w``/``_s``
    (layer 0) or ``moe`` (layers >= 1)."""
    input_ln: np.ndarray
    post_ln: np.ndarray
    proj: dict = field(default_factory=dict)  # q_w q_s k_w k_s v_w v_s o_w o_s
    dense: dict | None = None
    moe: MoeWeightsHost | None = None


@dataclass
class DecoderWeightsHost:
    hidden: int
    heads: int
    vocab: int
    layers: list
    final_norm: np.ndarray
    lm_w: np.ndarray
    lm_s: np.ndarray
    embed: np.ndarray  # [vocab, hidden] f32
    norm_topk_prob: bool = False  # moe.rs:73
    routed_scaling_factor: float = 1.0  # moe.rs:70


def rope_table(positions, head_dim: int = HEAD_DIM, theta: float = ROPE_THETA):
    """``RopeTable::build`` (decoder.rs:171-213) -> (cos, sin), each
    ``[len(positions), head_dim]`` f32, built by ``focr_rope_table``."""
    pos = np.ascontiguousarray(positions, dtype=np.uint64)
    n = pos.size
    c = np.empty((n, head_dim), np.float32)
    s = np.empty((n, head_dim), np.float32)
    check(lib.focr_rope_table(pos.ctypes.data, n, head_dim, float(theta), c.ctypes.data,
                              s.ctypes.data))
    return c, s


def _p(t):
    return t.data_ptr()


class DecoderI8:
    """Device-resident int8 decoder (weights uploaded once) with one R-SWA
    cache per layer: reference block ``[heads, max_prefill, head_dim]`` and
    ring ``[heads, 128, head_dim]`` for K and V."""

    def __init__(self, W: DecoderWeightsHost, max_prefill: int, device: str = "cuda",
                 max_batch: int = 1):
        import torch

        from .lmhead import LmHeadShard
        from .moe import MoeLayer

        self.W = W
        self.hidden, self.heads, self.vocab = W.hidden, W.heads, W.vocab
        self.dim = W.heads * HEAD_DIM
        self.max_prefill = max_prefill
        self.dev = torch.device(device)
        self._torch = torch

        def up(a):
            return torch.from_numpy(np.ascontiguousarray(a)).to(self.dev)

        self.layers = []
        for L in W.layers:
            d = {"input_ln": up(L.input_ln), "post_ln": up(L.post_ln)}
            for r in ("q", "k", "v", "o"):
                d[r + "_w"], d[r + "_s"] = up(L.proj[r + "_w"]), up(L.proj[r + "_s"])
            # fused q|k|v rows for the decode GEMV (fuse_qkv, decoder.rs:1951):
            # each output row is an independent dot, so byte-identical
            d["qkv_w"] = torch.cat([d["q_w"], d["k_w"], d["v_w"]]).contiguous()
            d["qkv_s"] = torch.cat([d["q_s"], d["k_s"], d["v_s"]]).contiguous()
            if L.dense is not None:
                d["inter"] = L.dense["gate_w"].shape[0]
                d["gu_w"] = up(np.concatenate([L.dense["gate_w"], L.dense["up_w"]]))
                d["gu_s"] = up(np.concatenate([L.dense["gate_s"], L.dense["up_s"]]))
                d["down_w"], d["down_s"] = up(L.dense["down_w"]), up(L.dense["down_s"])
            else:
                d["moe"] = MoeLayer(L.moe, max_tokens=max(max_prefill, max_batch),
                                    norm_topk_prob=W.norm_topk_prob,
                                    routed_scaling_factor=W.routed_scaling_factor)
            z = dict(dtype=torch.float32, device=self.dev)
            d["ref_k"] = torch.zeros((self.heads, max_prefill, HEAD_DIM), **z)
            d["ref_v"] = torch.zeros((self.heads, max_prefill, HEAD_DIM), **z)
            d["ring_k"] = torch.zeros((self.heads, RING_WINDOW, HEAD_DIM), **z)
            d["ring_v"] = torch.zeros((self.heads, RING_WINDOW, HEAD_DIM), **z)
            self.layers.append(d)
        self.final_norm = up(W.final_norm)
        self.head = LmHeadShard(W.lm_w, W.lm_s, row_begin=0, max_tokens=max(1, max_batch))
        self.embed = up(W.embed)
        self.prefill_len = None
        self.ring_len = 0
        self.ring_pos = 0

    def close(self):
        for d in self.layers:
            if "moe" in d:
                d["moe"].close()
        self.head.close()

    # -- device ops ---------------------------------------------------------------
    def _stream(self):
        return self._torch.cuda.current_stream().cuda_stream

    def _empty(self, *shape):
        return self._torch.empty(shape, dtype=self._torch.float32, device=self.dev)

    def _norm(self, x, w):
        y = self._empty(*x.shape)
        check(lib.focr_rms_norm(_p(x), x.shape[0], x.shape[1], _p(w), RMS_NORM_EPS, _p(y),
                                MEM_DEVICE, self._stream()))
        return y

    def _linear(self, x, w, s, te: bool):
        y = self._empty(x.shape[0], w.shape[0])
        check(lib.focr_linear_i8(_p(x), x.shape[0], x.shape[1], _p(w), _p(s), w.shape[0],
                                 int(te), _p(y), MEM_DEVICE, self._stream()))
        return y

    def _add_norm(self, a, b, w):
        """(a + b, rms_norm(a + b) * w) in one kernel."""
        h = self._empty(*a.shape)
        y = self._empty(*a.shape)
        check(lib.focr_add_rms_norm(_p(a), _p(b), a.shape[0], a.shape[1], _p(w), RMS_NORM_EPS,
                                    _p(h), _p(y), self._stream()))
        return h, y

    def _add(self, a, b):
        y = self._empty(*a.shape)
        check(lib.focr_add(_p(a), _p(b), a.numel(), _p(y), MEM_DEVICE, self._stream()))
        return y

    def _rope(self, x, cos_t, sin_t, cols=None):
        check(lib.focr_rope_apply(_p(x), x.shape[0], cols or x.shape[1], HEAD_DIM, _p(cos_t),
                                  _p(sin_t), MEM_DEVICE, self._stream()))

    def _dense(self, d, x, te: bool):
        gu = self._linear(x, d["gu_w"], d["gu_s"], te)
        act = self._empty(x.shape[0], d["inter"])
        check(lib.focr_swiglu(_p(gu), x.shape[0], d["inter"], _p(act), MEM_DEVICE,
                              self._stream()))
        return self._linear(act, d["down_w"], d["down_s"], te)

    # -- reference entry points -----------------------------------------------------
    def prefill(self, embeds):
        """``prefill_with_cache_i8``: ``embeds`` ``[seq, hidden]`` (device f32)
        -> final hidden states ``[seq, hidden]``; resets every layer's cache."""
        torch = self._torch
        seq = embeds.shape[0]
        if not 0 < seq <= self.max_prefill:
            raise ValueError(f"prefill seq {seq} outside (0, {self.max_prefill}]")
        c, s = rope_table(np.arange(seq))
        cos_t, sin_t = torch.from_numpy(c).to(self.dev), torch.from_numpy(s).to(self.dev)
        x = embeds.contiguous()
        mlp = None
        for d in self.layers:
            if mlp is None:
                normed = self._norm(x, d["input_ln"])
            else:  # x = h + mlp of the previous layer, fused with this norm
                x, normed = self._add_norm(h, mlp, d["input_ln"])
            q = self._linear(normed, d["q_w"], d["q_s"], True)
            k = self._linear(normed, d["k_w"], d["k_s"], True)
            v = self._linear(normed, d["v_w"], d["v_s"], True)
            self._rope(q, cos_t, sin_t)
            self._rope(k, cos_t, sin_t)
            d["ref_k"][:, :seq].copy_(k.view(seq, self.heads, HEAD_DIM).transpose(0, 1))
            d["ref_v"][:, :seq].copy_(v.view(seq, self.heads, HEAD_DIM).transpose(0, 1))
            ctx = self._empty(seq, self.dim)
            check(lib.focr_attention_prefill(_p(q), _p(k), _p(v), seq, self.heads, HEAD_DIM,
                                             _p(ctx), MEM_DEVICE, self._stream()))
            h, normed2 = self._add_norm(x, self._linear(ctx, d["o_w"], d["o_s"], True),
                                        d["post_ln"])
            if "moe" in d:
                mlp, _, _ = d["moe"].prefill(normed2)
            else:
                mlp = self._dense(d, normed2, True)
        x = self._add(h, mlp)
        self.prefill_len = seq
        self.ring_len = 0
        self.ring_pos = 0
        return x

    def _ring_slot(self) -> int:
        """``RingCache::write_decode_step`` slot rule (rswa.rs:467-493)."""
        if self.ring_len < RING_WINDOW:
            slot = self.ring_len
            self.ring_len += 1
            self.ring_pos = self.ring_len % RING_WINDOW
        else:
            slot = self.ring_pos
            self.ring_pos = (self.ring_pos + 1) % RING_WINDOW
        return slot

    def decode_step(self, token_embed, position: int):
        """``decode_step_with_cache_i8``: ``token_embed`` ``[1, hidden]`` ->
        hidden ``[1, hidden]``; writes this step's K/V into every ring."""
        torch = self._torch
        if self.prefill_len is None:
            raise RuntimeError("rswa: write_decode_step before record_prefill")
        c, s = rope_table([position])
        cos_t, sin_t = torch.from_numpy(c).to(self.dev), torch.from_numpy(s).to(self.dev)
        slot = self._ring_slot()
        D = self.dim
        x = token_embed.contiguous()
        mlp = None
        for d in self.layers:
            if mlp is None:
                normed = self._norm(x, d["input_ln"])
            else:
                x, normed = self._add_norm(h, mlp, d["input_ln"])
            qkv = self._linear(normed, d["qkv_w"], d["qkv_s"], False)
            self._rope(qkv, cos_t, sin_t, cols=2 * D)  # q and k: one row, 2 * heads heads
            d["ring_k"][:, slot].copy_(qkv[0, D:2 * D].view(self.heads, HEAD_DIM))
            d["ring_v"][:, slot].copy_(qkv[0, 2 * D:].view(self.heads, HEAD_DIM))
            ctx = self._empty(1, D)
            check(lib.focr_attention_decode(
                _p(qkv), _p(d["ref_k"]), _p(d["ref_v"]), self.prefill_len, self.max_prefill,
                _p(d["ring_k"]), _p(d["ring_v"]), self.ring_len, RING_WINDOW, self.heads,
                HEAD_DIM, _p(ctx), MEM_DEVICE, self._stream()))
            h, normed2 = self._add_norm(x, self._linear(ctx, d["o_w"], d["o_s"], False),
                                        d["post_ln"])
            if "moe" in d:
                mlp, _, _ = d["moe"].decode(normed2)
            else:
                mlp = self._dense(d, normed2, False)
        return self._add(h, mlp)

    def lm_head_top1(self, hidden_row):
        """``lm_head_cached_i8`` + ``argmax_row`` on a ``[1, hidden]`` row ->
        (best logit, token id) as device tensors."""
        normed = self._norm(hidden_row, self.final_norm)
        bv, bi, _ = self.head.top1(normed)
        return bv, bi

    def generate(self, embeds, n_tokens: int) -> np.ndarray:
        """Greedy decode of ``n_tokens`` after prefilling ``embeds``."""
        h = self.prefill(embeds)
        seq = embeds.shape[0]
        out = np.empty(n_tokens, np.int64)
        for i in range(n_tokens):
            _, bi = self.lm_head_top1(h[-1:])
            tok = int(bi.item())
            out[i] = tok
            if i + 1 == n_tokens:
                break
            h = self.decode_step(self.embed[tok:tok + 1], seq + i)
        return out

    # -- graph-replayed greedy decode ---------------------------------------------
    def _step_dev(self):
        """One decode step driven by the device state: prologue (record the
        previous token, advance position and ring cursor, gather the
        embedding), every layer, final norm and lm-head argmax into
        ``self._tok``.  Capturable: no host-varying argument."""
        st = self._stream()
        D = self.dim
        check(lib.focr_decode_prologue(_p(self._state), _p(self._tok), _p(self.embed), self.vocab,
                                       self.hidden, RING_WINDOW, _p(self._tokens),
                                       self._tokens.numel(), _p(self._x), st))
        x = self._x
        mlp = None
        for d in self.layers:
            # residual add + input RMSNorm + q|k|v projection, one launch
            qkv = self._empty(1, 3 * D)
            if mlp is None:
                check(lib.focr_rms_norm_linear_i8(_p(x), None, self.hidden, _p(d["input_ln"]),
                                                  RMS_NORM_EPS, None, _p(d["qkv_w"]),
                                                  _p(d["qkv_s"]), 3 * D, _p(qkv), st))
            else:
                x = self._empty(1, self.hidden)
                check(lib.focr_rms_norm_linear_i8(_p(h), _p(mlp), self.hidden, _p(d["input_ln"]),
                                                  RMS_NORM_EPS, _p(x), _p(d["qkv_w"]),
                                                  _p(d["qkv_s"]), 3 * D, _p(qkv), st))
            # RoPE of q and k, then k and v into the ring slot: one launch
            check(lib.focr_rope_ring_at(_p(qkv), self.heads, HEAD_DIM, _p(self._cos),
                                        _p(self._sin), _p(d["ring_k"]), _p(d["ring_v"]),
                                        RING_WINDOW, _p(self._state), st))
            ctx = self._empty(1, D)
            check(lib.focr_attention_decode_at(
                _p(qkv), _p(d["ref_k"]), _p(d["ref_v"]), self.prefill_len, self.max_prefill,
                _p(d["ring_k"]), _p(d["ring_v"]), RING_WINDOW, self.heads, HEAD_DIM,
                _p(self._state), _p(ctx), st))
            h, normed2 = self._add_norm(x, self._linear(ctx, d["o_w"], d["o_s"], False),
                                        d["post_ln"])
            if "moe" in d:
                mlp, _, _ = d["moe"].decode(normed2)
            else:
                mlp = self._dense(d, normed2, False)
        _, normed = self._add_norm(h, mlp, self.final_norm)
        check(lib.focr_lmhead_top1(self.head._h, _p(normed), 1, _p(self._bv), _p(self._tok), None,
                                   MEM_DEVICE, st))

    def _head_top1(self, row):
        normed = self._norm(row, self.final_norm)
        check(lib.focr_lmhead_top1(self.head._h, _p(normed), 1, _p(self._bv), _p(self._tok), None,
                                   MEM_DEVICE, self._stream()))

    def generate_graph(self, embeds, n_tokens: int, use_graph: bool = True,
                       timer: list | None = None) -> np.ndarray:
        """:meth:`generate` with the decode loop on the device: the step is
        captured once in a CUDA graph and replayed per token; tokens are
        recorded on the device and read back once at the end.  With `timer`
        (a list) the call appends (start event, end event, replayed steps)
        bracketing the graph replays on the current stream."""
        torch = self._torch
        from ._lib import STATE_NEXT_POS, STATE_WORDS

        seq = embeds.shape[0]
        key = (seq, n_tokens)
        if getattr(self, "_graph_key", None) != key:
            # buffers the captured step points at: fixed for a (seq, n_tokens)
            c, s = rope_table(np.arange(seq + n_tokens))
            self._cos, self._sin = torch.from_numpy(c).to(self.dev), torch.from_numpy(s).to(self.dev)
            self._state = torch.zeros(STATE_WORDS, dtype=torch.int32, device=self.dev)
            self._tok = torch.zeros(1, dtype=torch.int32, device=self.dev)
            self._bv = torch.zeros(1, dtype=torch.float32, device=self.dev)
            self._x = self._empty(1, self.hidden)
            self._tokens = torch.zeros(n_tokens, dtype=torch.int32, device=self.dev)
            self._graph, self._graph_key = None, key
        st0 = np.zeros(STATE_WORDS, np.int32)
        st0[STATE_NEXT_POS] = seq
        self._state.copy_(torch.from_numpy(st0))
        h = self.prefill(embeds)
        self._head_top1(h[-1:])
        steps = n_tokens - 1
        if steps > 0:
            self._step_dev()  # eager: first step, and one-time kernel attributes
        if steps > 1:
            if use_graph:
                g = self._graph
                if g is None:
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        self._step_dev()
                    self._graph = g
                if timer is not None:
                    t0 = torch.cuda.Event(enable_timing=True)
                    t1 = torch.cuda.Event(enable_timing=True)
                    t0.record()
                for _ in range(steps - 1):
                    g.replay()
                if timer is not None:
                    t1.record()
                    timer.append((t0, t1, steps - 1))
            else:
                for _ in range(steps - 1):
                    self._step_dev()
        self._tokens[n_tokens - 1:].copy_(self._tok)
        out = self._tokens.cpu().numpy().astype(np.int64)
        st = self._state.cpu().numpy()
        if st[6]:
            raise RuntimeError("decode: token id outside the embedding table")
        self.ring_len, self.ring_pos = int(st[1]), int(st[2])
        return out


def _np_ptr(a):
    return None if a is None else a.ctypes.data


class DecoderLib:
    """The whole decoder as one library object (``focr_decoder_*``): weights
    uploaded, caches and activations allocated and the decode step captured
    in a CUDA graph by ``libfocr_cuda.so`` itself -- the path a host without
    PyTorch (the reference's Rust engine over its FFI crate) drives.  Host
    numpy inputs and outputs."""

    def __init__(self, W: DecoderWeightsHost, max_prefill: int):
        self.W = W
        self.hidden, self.vocab = W.hidden, W.vocab
        keep = []

        def arr(a, dt):
            a = np.ascontiguousarray(a, dtype=dt)
            keep.append(a)
            return a.ctypes.data

        moe_shape = next((L.moe for L in W.layers if L.moe is not None), None)
        mc = MoeConfig()
        if moe_shape is not None:
            mc = MoeConfig(moe_shape.hidden, moe_shape.inter, moe_shape.n_experts, moe_shape.topk,
                           moe_shape.shared_inter, int(W.norm_topk_prob),
                           float(W.routed_scaling_factor), moe_shape.group,
                           moe_shape.expert_begin, moe_shape.expert_count, max_prefill)
        cfg = DecoderConfig(W.hidden, W.heads, HEAD_DIM, len(W.layers), W.vocab, max_prefill,
                            RING_WINDOW, ROPE_THETA, RMS_NORM_EPS, mc)
        layers = (DecoderLayerWeights * len(W.layers))()
        moe_w = []
        for i, L in enumerate(W.layers):
            lw = layers[i]
            lw.input_ln, lw.post_ln = arr(L.input_ln, np.float32), arr(L.post_ln, np.float32)
            for r in ("q", "k", "v", "o"):
                setattr(lw, r + "_w", arr(L.proj[r + "_w"], np.int8))
                setattr(lw, r + "_s", arr(L.proj[r + "_s"], np.float32))
            if L.moe is not None:
                mw = MoeWeights()
                mw.router = arr(L.moe.router, np.float32)
                for name, a in L.moe.arrays.items():
                    setattr(mw, name, _np_ptr(a))
                    keep.append(a)
                moe_w.append(mw)
                lw.moe = C.cast(C.pointer(mw), C.c_void_p)
            else:
                lw.dense_inter = L.dense["gate_w"].shape[0]
                for n in ("gate", "up", "down"):
                    setattr(lw, n + "_w", arr(L.dense[n + "_w"], np.int8))
                    setattr(lw, n + "_s", arr(L.dense[n + "_s"], np.float32))
        wt = DecoderWeights(layers, arr(W.final_norm, np.float32), arr(W.lm_w, np.int8),
                            arr(W.lm_s, np.float32), arr(W.embed, np.float32))
        h = C.c_void_p()
        check(lib.focr_decoder_create(C.byref(cfg), C.byref(wt), C.byref(h)))
        self._h = h
        del keep, moe_w

    def close(self):
        if getattr(self, "_h", None):
            lib.focr_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def prefill(self, embeds: np.ndarray) -> np.ndarray:
        e = np.ascontiguousarray(embeds, dtype=np.float32)
        out = np.empty_like(e)
        check(lib.focr_decoder_prefill(self._h, e.ctypes.data, e.shape[0], out.ctypes.data,
                                       MEM_HOST, None))
        return out

    def generate(self, embeds: np.ndarray, n_tokens: int) -> np.ndarray:
        e = np.ascontiguousarray(embeds, dtype=np.float32)
        toks = np.empty(n_tokens, np.int32)
        check(lib.focr_decoder_generate(self._h, e.ctypes.data, e.shape[0], n_tokens,
                                        toks.ctypes.data, MEM_HOST, None))
        return toks.astype(np.int64)
