"""Continuous-batch scheduler (CPU): the reference's scheduler tests
(native_engine/batch_scheduler.rs:535-760) restated with a weights-free step,
and the decoder batch step composed over per-stream oracle decoders, which
must reproduce each stream's single-stream greedy sequence."""
import numpy as np
import pytest

from franken_ocr_b200.batch import (BatchScheduler, DecoderBatchStep, PageStream, StreamOut,
                                    admission_order)


class MockStep:
    """hidden = (tag, eos_after); token = emitted count so far; EOS on the
    eos_after-th token (0 = never)."""

    def __init__(self):
        self.active_sizes = []
        self.slot_seen = []

    def step(self, slots):
        self.active_sizes.append(len(slots))
        out = []
        for s in slots:
            tag, eos_after = s.hidden
            self.slot_seen.append((s.slot_index, tag))
            n = len(s.history)
            out.append(StreamOut(n, eos_after > 0 and n + 1 >= eos_after, s.hidden))
        return out


def stream(i, eos_after, prefill_len=0):
    return PageStream(i, prefill_len, [], (i, eos_after))


def test_each_stream_emits_exactly_eos_after_tokens():
    toks = BatchScheduler(3, 100).run([stream(i, e) for i, e in enumerate([1, 4, 2, 7])], MockStep())
    assert [len(t) for t in toks] == [1, 4, 2, 7]
    assert toks[3] == list(range(7))


def test_outputs_resorted_to_input_order_despite_shuffled_submission():
    streams = [stream(i, i + 1) for i in (3, 0, 2, 1)]
    toks = BatchScheduler(2, 100).run(streams, MockStep())
    assert [len(t) for t in toks] == [1, 2, 3, 4]


def test_one_live_forward_and_active_set_bounded_with_backfill():
    sched = BatchScheduler(2, 100)
    m = MockStep()
    sched.run([stream(i, e) for i, e in enumerate([1, 3, 2, 2, 1])], m)
    st = sched.stats()
    assert st.max_concurrent_forwards == 1
    assert st.max_active == 2 and max(m.active_sizes) == 2
    assert st.total_steps == len(m.active_sizes)
    # backfill: after stream 0 retires on step 1, stream 2 joins step 2
    assert m.active_sizes[:2] == [2, 2]


def test_batch_size_one_serializes_all_streams():
    m = MockStep()
    toks = BatchScheduler(1, 100).run([stream(i, 3) for i in range(3)], m)
    assert toks == [[0, 1, 2]] * 3 and set(m.active_sizes) == {1}


def test_max_length_retires_unbounded_streams():
    toks = BatchScheduler(4, 5).run([stream(i, 0) for i in range(2)], MockStep())
    assert toks == [[0, 1, 2, 3, 4]] * 2


def test_empty_input_yields_empty_output():
    sched = BatchScheduler(4, 5)
    assert sched.run([], MockStep()) == [] and sched.stats().total_steps == 0


def test_batch_size_is_clamped():
    assert BatchScheduler(0, 1).batch_size == 1
    assert BatchScheduler(10 ** 6, 1).batch_size == 64


def test_slot_index_identifies_the_stream_through_retire_and_backfill():
    m = MockStep()
    BatchScheduler(2, 100).run([stream(i, e) for i, e in enumerate([2, 1, 3, 1])], m)
    assert all(slot == tag for slot, tag in m.slot_seen)


def test_pack_admission_is_a_stable_length_grouping():
    streams = [stream(i, 1, p) for i, p in enumerate([30, 10, 30, 5, 10])]
    assert admission_order(streams, False) == [0, 1, 2, 3, 4]
    assert admission_order(streams, True) == [3, 1, 4, 0, 2]
    toks = BatchScheduler(2, 3).run(streams, MockStep(), pack=True)
    assert toks == [[0]] * 5


class OracleStreams:
    """Per-slot oracle decoders behind the batch-decoder interface."""

    def __init__(self, oracle, W, n):
        self.O, self.W, self.vocab = oracle, W, W.vocab
        self.dec = [oracle.DecoderOracle(W) for _ in range(n)]

    def prefill_stream(self, slot, e):
        return self.dec[slot].prefill(e)[-1]

    def lm_head_argmax(self, hiddens):
        return [self.O.argmax_row(self.dec[0].lm_head(h)) for h in hiddens]

    def decode_streams(self, ids, toks, pos):
        return [self.dec[s].decode_step(self.W.embed[t], p)[0] for s, t, p in zip(ids, toks, pos)]


def test_decoder_batch_step_reproduces_single_stream_sequences(oracle):
    from franken_ocr_b200 import synth

    W = synth.decoder_model(21, layers=2, n_experts=4, topk=2, dense_inter=128, vocab=256,
                            shared_inter=64)
    lens, n_tok = [5, 9, 3], 6
    embeds = [synth.prompt_embeds(21 + i, n, W.hidden) for i, n in enumerate(lens)]
    want = [oracle.DecoderOracle(W).generate(e, n_tok) for e in embeds]
    dec = OracleStreams(oracle, W, 3)
    streams = [PageStream(i, lens[i], [], dec.prefill_stream(i, embeds[i])) for i in range(3)]
    got = BatchScheduler(2, n_tok).run(streams, DecoderBatchStep(dec, eos_token_id=-1))
    for g, w in zip(got, want):
        assert np.array_equal(np.array(g), w)


def test_batch_step_rejects_out_of_vocab_tokens():
    class Bad:
        vocab = 4

        def lm_head_argmax(self, h):
            return [7]

        def decode_streams(self, *a):
            raise AssertionError("not reached")

    slot = PageStream(0, 1, [], None)
    with pytest.raises(RuntimeError, match="outside embed vocab"):
        BatchScheduler(1, 1).run([slot], DecoderBatchStep(Bad()))
