"""Regenerate ``decoder_config3_greedy256.json``: the CPU oracle's greedy
tokens for the config-3 decoder (12 layers, seed 3, a 1024-token prefill of
N(0,1) embeddings, then 256 greedy tokens at batch 1).

The oracle is the scalar C restatement of the reference's int8 decoder loop
(``oracle.oracle.DecoderOracle``: prefill_with_cache_i8, decode_step_with_cache_i8,
lm_head_cached_i8 + argmax_row, the greedy loop of generate_cached_i8 in
native_engine/mod.rs:1860-1898).  It runs single-threaded here, so the
fixture does not depend on the threaded CPU tier.  The fixture also records,
per generated token, the f64 sum and L2 norm of the final hidden row the
token was read from, and the winning logit, for a tolerance check of the
hidden state beside the exact token check.

Usage: python tests/golden/make_decoder_golden.py [prefill] [n_tokens]
(takes tens of minutes on one core at the full size).
"""
import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))


def main(prefill: int = 1024, n_tokens: int = 256, seed: int = 3) -> None:
    from franken_ocr_b200 import synth
    from oracle import oracle as O

    W = synth.decoder_model(seed)
    e = synth.prompt_embeds(seed, prefill)
    D = O.DecoderOracle(W)
    t0 = time.time()
    h = D.prefill(e)
    t_pre = time.time() - t0
    toks, sums, norms, logits = [], [], [], []
    for i in range(n_tokens):
        row = h[-1].astype(np.float64)
        sums.append(float(row.sum()))
        norms.append(float(np.sqrt((row * row).sum())))
        lg = D.lm_head(h[-1])
        tok = O.argmax_row(lg)
        toks.append(int(tok))
        logits.append(float(lg[tok]))
        if i + 1 < n_tokens:
            h = D.decode_step(W.embed[tok], prefill + i)
    out = {
        "what": "greedy tokens of the CPU oracle decoder (scalar restatement)",
        "model": "synth.decoder_model(seed)", "seed": seed, "layers": len(W.layers),
        "prefill_tokens": prefill, "prompt": "synth.prompt_embeds(seed, prefill_tokens)",
        "n_tokens": n_tokens, "tokens": toks, "hidden_sum": sums, "hidden_l2": norms,
        "top1_logit": logits,
        "oracle_seconds": {"prefill": round(t_pre, 1), "total": round(time.time() - t0, 1)},
    }
    name = f"decoder_config3_greedy{n_tokens}.json" if prefill == 1024 else \
        f"decoder_seed{seed}_p{prefill}_greedy{n_tokens}.json"
    (HERE / name).write_text(json.dumps(out, indent=0) + "\n")
    print(name, toks[:16], out["oracle_seconds"])


if __name__ == "__main__":
    a = [int(v) for v in sys.argv[1:]]
    main(*a)
