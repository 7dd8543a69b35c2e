"""Continuous-batch greedy decode: the scheduler and its decoder step.

Mirrors native_engine/batch_scheduler.rs:

* :class:`BatchScheduler` -- ``BatchScheduler::run`` (batch_scheduler.rs:298-380):
  up to ``batch_size`` streams are active in one forward; a stream retires on
  EOS or after ``max_length`` emitted tokens and the active set is backfilled
  from the pending queue (submission order, or length-grouped when ``pack``,
  ``admission_order`` :109-117); outputs are re-sorted to input order.  Exactly
  one forward is live at a time (``stats().max_concurrent_forwards``).
* :class:`DecoderBatchStep` -- ``DecoderBatchStep::step`` (:433-500): the
  batched lm-head + greedy argmax over the active streams, then one batched
  decode step of exactly those streams (``batched_decode_step_i8_streams``,
  decoder.rs:2812-2933), each addressing its own cache slot.
* :class:`BatchedDecoderI8` -- the device side: one shared weight set
  (a :class:`~franken_ocr_b200.decoder.DecoderI8`) and per-stream R-SWA caches.
  Projections and the lm-head run at M = active streams (each output row is
  the row a single-stream call computes, bit for bit: per-row activation
  quantisation, exact int32 dots); RoPE at each stream's own position, the
  ring write and decode attention stay per stream; the MoE layer decodes the
  M rows with per-row routing.

Sampling is greedy ``argmax_row`` with EOS = token 1 (decoder.rs config
``EOS_TOKEN_ID``); the n-gram bans of ``sampler::batched_decode_step`` are
product policy and not part of this path.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

from ._lib import MEM_DEVICE, check, lib
from .decoder import HEAD_DIM, RING_WINDOW, DecoderI8, rope_table

EOS_TOKEN_ID = 1
MAX_BATCH_SIZE = 64


@dataclass
class PageStream:
    """One in-flight stream (batch_scheduler.rs:123-166)."""
    input_index: int
    prefill_len: int
    prompt_ids: list
    last_hidden: object  # [1, hidden] row (device tensor or numpy)
    position: int = -1
    generated: list = field(default_factory=list)
    prompt_len: int = 0
    done: bool = False
    eos: bool = False

    def __post_init__(self):
        if self.position < 0:
            self.position = self.prefill_len
        self.generated = list(self.prompt_ids)
        self.prompt_len = len(self.prompt_ids)

    def emitted(self) -> list:
        return self.generated[self.prompt_len:]


@dataclass
class StreamSlot:
    slot_index: int  # index into the submitted streams = the stream's cache slot
    history: list
    hidden: object
    position: int


@dataclass
class StreamOut:
    token: int
    is_eos: bool
    new_hidden: object


@dataclass
class SchedulerStats:
    max_concurrent_forwards: int
    max_active: int
    total_steps: int


def admission_order(streams, pack: bool) -> list:
    """Submission order, or a stable sort by prefill length when ``pack``."""
    order = list(range(len(streams)))
    if pack:
        order.sort(key=lambda i: streams[i].prefill_len)
    return order


class BatchScheduler:
    def __init__(self, batch_size: int, max_length: int):
        self.batch_size = max(1, min(int(batch_size), MAX_BATCH_SIZE))
        self.max_length = max_length
        self._live = 0
        self._max_live = 0
        self._max_active = 0
        self._steps = 0

    def stats(self) -> SchedulerStats:
        return SchedulerStats(self._max_live, self._max_active, self._steps)

    @staticmethod
    def _admit(active: list, pending: deque, cap: int) -> None:
        while len(active) < cap and pending:
            active.append(pending.popleft())

    def run(self, streams: list, step, pack: bool = False) -> list:
        """Drive ``streams`` to completion through ``step`` (an object with
        ``step(slots) -> [StreamOut]``); returns each stream's emitted tokens in
        ``input_index`` order."""
        pending = deque(admission_order(streams, pack))
        active: list = []
        self._admit(active, pending, self.batch_size)
        while active:
            self._max_active = max(self._max_active, len(active))
            slots = [StreamSlot(i, streams[i].generated, streams[i].last_hidden,
                                streams[i].position) for i in active]
            self._live += 1
            self._max_live = max(self._max_live, self._live)
            try:
                outs = step.step(slots)
            finally:
                self._live -= 1
            self._steps += 1
            if len(outs) != len(active):
                raise RuntimeError(f"batch step returned {len(outs)} outputs for "
                                   f"{len(active)} active streams")
            retire = []
            for k, (i, out) in enumerate(zip(active, outs)):
                s = streams[i]
                s.generated.append(int(out.token))
                s.position += 1
                if out.is_eos or len(s.emitted()) >= self.max_length:
                    s.done, s.eos = True, bool(out.is_eos)
                    retire.append(k)
                else:
                    s.last_hidden = out.new_hidden
            for k in reversed(retire):
                active.pop(k)
            self._admit(active, pending, self.batch_size)
        order = sorted(range(len(streams)), key=lambda i: streams[i].input_index)
        return [streams[i].emitted() for i in order]


class DecoderBatchStep:
    """``DecoderBatchStep::step``: greedy tokens from the active hiddens, then
    one decode step of the active streams.  ``decoder`` provides
    ``lm_head_argmax(hiddens) -> token ids`` and
    ``decode_streams(stream_ids, token_ids, positions) -> new hiddens``."""

    def __init__(self, decoder, eos_token_id: int = EOS_TOKEN_ID):
        self.decoder = decoder
        self.eos = eos_token_id

    def step(self, slots: list) -> list:
        toks = [int(t) for t in self.decoder.lm_head_argmax([s.hidden for s in slots])]
        vocab = self.decoder.vocab
        for t in toks:
            if not 0 <= t < vocab:
                raise RuntimeError(f"batch step: token id {t} outside embed vocab {vocab}")
        new = self.decoder.decode_streams([s.slot_index for s in slots], toks,
                                          [s.position for s in slots])
        return [StreamOut(t, t == self.eos, h) for t, h in zip(toks, new)]


class BatchedDecoderI8:
    """Shared int8 weights + ``n_streams`` R-SWA cache slots
    (``BatchedRingCache``, rswa.rs:620-700): slot ``i`` holds stream ``i``'s
    reference block ``[heads, max_prefill, 128]`` and ring ``[heads, 128, 128]``
    for every layer."""

    def __init__(self, W, n_streams: int, max_prefill: int, device: str = "cuda"):
        import torch

        self._torch = torch
        self.core = DecoderI8(W, max_prefill=max_prefill, device=device, max_batch=n_streams)
        self.n_streams = n_streams
        self.vocab, self.hidden, self.heads = W.vocab, W.hidden, W.heads
        self.dim = W.heads * HEAD_DIM
        self.max_prefill = max_prefill
        dev = self.core.dev
        z = dict(dtype=torch.float32, device=dev)
        L = len(self.core.layers)
        shp_ref = (L, n_streams, W.heads, max_prefill, HEAD_DIM)
        shp_ring = (L, n_streams, W.heads, RING_WINDOW, HEAD_DIM)
        self.ref_k, self.ref_v = torch.zeros(shp_ref, **z), torch.zeros(shp_ref, **z)
        self.ring_k, self.ring_v = torch.zeros(shp_ring, **z), torch.zeros(shp_ring, **z)
        self.prefill_len = [0] * n_streams
        self.ring_len = [0] * n_streams
        self.ring_pos = [0] * n_streams

    def close(self):
        self.core.close()

    def prefill_stream(self, slot: int, embeds):
        """``prefill_with_cache_i8`` for one stream into cache slot ``slot``;
        returns the last hidden row ``[1, hidden]``."""
        if not 0 <= slot < self.n_streams:
            raise ValueError(f"stream slot {slot} outside [0, {self.n_streams})")
        h = self.core.prefill(embeds)
        seq = embeds.shape[0]
        for li, d in enumerate(self.core.layers):
            self.ref_k[li, slot, :, :seq].copy_(d["ref_k"][:, :seq])
            self.ref_v[li, slot, :, :seq].copy_(d["ref_v"][:, :seq])
        self.prefill_len[slot], self.ring_len[slot], self.ring_pos[slot] = seq, 0, 0
        return h[-1:].clone()

    def lm_head_argmax(self, hiddens) -> list:
        """``batched_lm_head_i8`` + ``argmax_row`` per row (decoder.rs:2943)."""
        torch = self._torch
        core = self.core
        x = torch.cat([h.reshape(1, -1) for h in hiddens]).contiguous()
        normed = core._norm(x, core.final_norm)
        _, bi, _ = core.head.top1(normed)
        return bi.cpu().tolist()

    def _slot(self, sid: int) -> int:
        if self.ring_len[sid] < RING_WINDOW:
            slot = self.ring_len[sid]
            self.ring_len[sid] += 1
            self.ring_pos[sid] = self.ring_len[sid] % RING_WINDOW
        else:
            slot = self.ring_pos[sid]
            self.ring_pos[sid] = (slot + 1) % RING_WINDOW
        return slot

    def decode_streams(self, stream_ids, token_ids, positions) -> list:
        """``batched_decode_step_i8_streams``: advance the given cache slots one
        step with their tokens at their positions; returns the new hidden rows."""
        torch = self._torch
        core = self.core
        B = len(stream_ids)
        if not (B == len(token_ids) == len(positions)) or B == 0:
            raise ValueError("decode_streams: stream_ids, token_ids and positions must have the "
                             "same non-zero length")
        if len(set(stream_ids)) != B or any(not 0 <= s < self.n_streams for s in stream_ids):
            raise ValueError("decode_streams: stream ids must be distinct cache slots")
        for s in stream_ids:
            if self.prefill_len[s] == 0:
                raise RuntimeError("rswa: write_decode_step before record_prefill")
        dev = core.dev
        D, st = self.dim, core._stream()
        c, s_ = rope_table(positions)
        cos_t, sin_t = torch.from_numpy(c).to(dev), torch.from_numpy(s_).to(dev)
        slots = [self._slot(s) for s in stream_ids]
        sid_t = torch.tensor(stream_ids, device=dev)
        slot_t = torch.tensor(slots, device=dev)
        x = core.embed[torch.tensor(token_ids, device=dev)].contiguous()
        mlp = None
        for li, d in enumerate(core.layers):
            if mlp is None:
                normed = core._norm(x, d["input_ln"])
            else:
                x, normed = core._add_norm(h, mlp, d["input_ln"])
            qkv = core._linear(normed, d["qkv_w"], d["qkv_s"], False)
            q = qkv[:, :D].contiguous()
            k = qkv[:, D:2 * D].contiguous()
            core._rope(q, cos_t, sin_t)
            core._rope(k, cos_t, sin_t)
            # every stream writes its own ring slot (RingCache::write_decode_step)
            self.ring_k[li, sid_t, :, slot_t] = k.view(B, self.heads, HEAD_DIM)
            self.ring_v[li, sid_t, :, slot_t] = qkv[:, 2 * D:].reshape(B, self.heads, HEAD_DIM)
            ctx = core._empty(B, D)
            for j, sid in enumerate(stream_ids):
                check(lib.focr_attention_decode(
                    q[j].data_ptr(), self.ref_k[li, sid].data_ptr(),
                    self.ref_v[li, sid].data_ptr(), self.prefill_len[sid], self.max_prefill,
                    self.ring_k[li, sid].data_ptr(), self.ring_v[li, sid].data_ptr(),
                    self.ring_len[sid], RING_WINDOW, self.heads, HEAD_DIM, ctx[j].data_ptr(),
                    MEM_DEVICE, st))
            h, normed2 = core._add_norm(x, core._linear(ctx, d["o_w"], d["o_s"], False),
                                        d["post_ln"])
            if "moe" in d:
                mlp, _, _ = d["moe"].decode(normed2)
            else:
                mlp = core._dense(d, normed2, False)
        out = core._add(h, mlp)
        return [out[j:j + 1] for j in range(B)]
