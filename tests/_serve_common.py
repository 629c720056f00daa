"""Shared pieces of the continuous-batching tests: a small random model, the
serial restatement of serve.rs generate_completion on the oracle (the
expected tokens), and the request mix."""
import numpy as np

from hypno_b200 import synth
from oracle import oracle as orc

# head_dim 64, GQA group 2; with std 0.5 every greedy pick of request_mix has a
# top-2 margin of at least 2.4x the logits tolerance (1e-3 of max(1, max|logit|)),
# apart from the empty prompt's all-zero logits (an exact tie everywhere)
SMALL = dict(hidden=256, inter=512, heads=4, kv_heads=2, layers=2, vocab=512, theta=10000.0, max_pos=48,
             embed="fp32", lm_head="separate")


def small_image(seed=3):
    return synth.build_image(SMALL, seed=seed, std=0.5, quantize=orc.quantize_f32_to_q4_0)


def serial_generation(om, prompt, max_tokens, eos_id, max_pos, seen=None):
    """serve.rs:239-255 with the greedy pick (run.rs:234-238), one request
    alone on a fresh cache; stops with "length" where the next forward would
    need a position the cache does not have.  `seen` collects the logits each
    pick was made from."""
    kv = om.new_kv(max_pos)
    logits = orc.batch_forward(om, prompt, kv)
    toks, reason = [], "stop"
    for _ in range(max_tokens):
        if seen is not None:
            seen.append(logits)
        nxt = orc.greedy(logits)
        if eos_id is not None and nxt == eos_id:
            reason = "stop"
            break
        toks.append(nxt)
        if len(toks) == max_tokens:
            break
        if kv.seq_len() >= max_pos:
            reason = "length"
            break
        logits = orc.model_forward(om, nxt, kv)
    if max_tokens > 0 and len(toks) == max_tokens:
        reason = "length"
    return toks, reason


def request_mix(vocab, seed=11):
    """(prompt, max_tokens): ragged prompts, an empty prompt, max_tokens 0 and
    1, and one request that runs into the end of its slot."""
    g = np.random.Generator(np.random.PCG64(seed))
    lens_max = [(5, 12), (17, 9), (0, 6), (3, 0), (30, 8), (1, 1), (9, 20), (44, 30), (12, 7)]
    return [(g.integers(0, vocab, size=n).astype(np.uint32), m) for n, m in lens_max]
