"""GPU continuous batching: streams of different prompt lengths decoded
through the scheduler at batch width 2 (retire + backfill) produce each
stream's single-stream oracle tokens, and the M-row batched projections,
lm-head and MoE rows equal the single-stream computation."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_batched_decoder_matches_single_stream_oracle(cuda, oracle):
    import torch

    from franken_ocr_b200 import synth
    from franken_ocr_b200.batch import BatchedDecoderI8, BatchScheduler, DecoderBatchStep, PageStream

    W = synth.decoder_model(11, layers=3, n_experts=8, dense_inter=512, vocab=2048)
    lens, n_tok = [24, 40, 9], 12
    embeds = [synth.prompt_embeds(31 + i, n, W.hidden) for i, n in enumerate(lens)]
    want = [oracle.DecoderOracle(W).generate(e, n_tok) for e in embeds]
    B = BatchedDecoderI8(W, n_streams=3, max_prefill=max(lens))
    streams = [PageStream(i, lens[i], [], B.prefill_stream(i, torch.from_numpy(embeds[i]).cuda()))
               for i in range(3)]
    sched = BatchScheduler(2, n_tok)
    got = sched.run(streams, DecoderBatchStep(B, eos_token_id=-1))
    for i, (g, w) in enumerate(zip(got, want)):
        assert np.array_equal(np.array(g), w), (i, g, w)
    assert sched.stats().max_active == 2
    B.close()
