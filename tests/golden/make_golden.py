"""Generate golden vectors from the reference implementation itself.

    python tests/golden/make_golden.py <reference checkout>

Runs the reference's own beam-search loops (serving_engine.beam_search with a
catalog, llm.beam_search without) unmodified, on the mock engine of
oracle/ref_shim.py, and writes tests/golden/reference_beams.json: per case the
beams the reference asked the engine for at every step and its final sequences
with cumulative log-probs.  Cases cover float32 and bf16 logits, vLLM's raw
and processed log-prob modes (processed: the temperature the loop passes in
its SamplingParams divides the logits first), widths up to 16 beams, up to 4
prompts in one offline batch and vocabularies up to 8192.  The fixtures are
committed; the tests read only them (the reference checkout is not needed to
run the tests).
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_shim  # noqa: E402


def sid_catalog(n_items, levels, codebook, base, begin, end, seed):
    rng = np.random.default_rng(seed)
    seqs = set()
    while len(seqs) < n_items:
        codes = rng.integers(0, codebook, levels)
        seqs.add(tuple([begin] + [base + l * codebook + int(c) for l, c in enumerate(codes)] + [end]))
    return [list(s) for s in sorted(seqs)]


CASES = [
    dict(name="online_allowed_small", kind="online", mode="allowed", prompt=[5, 6, 7], beam_width=4, max_tokens=5,
         vocab=256, sigma=4.0, seed=0, catalog=dict(n_items=30, levels=3, codebook=8, base=210, begin=200, end=201,
                                                       seed=1), eos=255),
    dict(name="online_allowed_b8", kind="online", mode="allowed", prompt=[11, 12], beam_width=8, max_tokens=5,
         vocab=1024, sigma=3.0, seed=3, catalog=dict(n_items=300, levels=3, codebook=32, base=900, begin=890,
                                                        end=891, seed=2), eos=1023),
    dict(name="online_allowed_eos_child", kind="online", mode="allowed", prompt=[1], beam_width=3, max_tokens=5,
         vocab=128, sigma=2.0, seed=5, catalog=dict(n_items=12, levels=2, codebook=6, base=100, begin=90, end=91,
                                                       seed=4), eos=91),
    dict(name="offline_eos_lp1", kind="offline", prompts=[[1, 2], [3]], beam_width=3, max_tokens=4, vocab=64,
         sigma=2.0, seed=1, eos=7, length_penalty=1.0),
    dict(name="offline_eos_lp05", kind="offline", prompts=[[4], [5, 6, 7]], beam_width=4, max_tokens=5, vocab=48,
         sigma=1.5, seed=9, eos=3, length_penalty=0.5),
    # bf16 logits, processed log-probs with temperature, larger shapes.  bf16
    # rows hold many exactly equal values; among exactly equal scores the
    # reference's argpartition keeps an unspecified one, so the seeds below
    # give selections whose boundary holds no exact tie (the canonical order
    # among ties is checked against the oracle elsewhere).
    dict(name="online_bf16_b16_v8192", kind="online", mode="allowed", prompt=[21, 22, 23], beam_width=16,
         max_tokens=5, vocab=8192, sigma=4.0, seed=11, bf16=True,
         catalog=dict(n_items=3000, levels=3, codebook=128, base=7700, begin=7690, end=7691, seed=12), eos=8191),
    dict(name="online_processed_t07_b16", kind="online", mode="allowed", prompt=[31, 32], beam_width=16,
         max_tokens=5, vocab=8192, sigma=4.0, seed=13, processed=True, temperature=0.7,
         catalog=dict(n_items=3000, levels=3, codebook=128, base=7700, begin=7690, end=7691, seed=14), eos=8191),
    dict(name="online_processed_bf16_t13", kind="online", mode="allowed", prompt=[41], beam_width=8,
         max_tokens=5, vocab=4096, sigma=3.0, seed=15, bf16=True, processed=True, temperature=1.3,
         catalog=dict(n_items=800, levels=3, codebook=64, base=3800, begin=3790, end=3791, seed=16), eos=3791),
    dict(name="offline_bf16_r4_b16_v8192", kind="offline", prompts=[[1, 2], [3], [4, 5, 6], [7]], beam_width=16,
         max_tokens=4, vocab=8192, sigma=4.0, seed=18, bf16=True, eos=8191, length_penalty=1.0),
    dict(name="offline_processed_t07_r4", kind="offline", prompts=[[9], [10, 11], [12], [13, 14, 15]],
         beam_width=8, max_tokens=4, vocab=2048, sigma=2.0, seed=19, processed=True, temperature=0.7, eos=5,
         length_penalty=1.0),
]


def main(reference_root):
    out = []
    for c in CASES:
        rec = dict(c)
        if c["kind"] == "online":
            cat = sid_catalog(**c["catalog"])
            calls, beams = ref_shim.run_online(
                reference_root, c["prompt"], beam_width=c["beam_width"], max_tokens=c["max_tokens"], vocab=c["vocab"],
                sigma=c["sigma"], seed=c["seed"], bf16=c.get("bf16", False), catalog_seqs=cat,
                begin_token=c["catalog"]["begin"], end_token=c["catalog"]["end"], eos_token_id=c["eos"],
                ignore_eos=False, mode=c["mode"], processed=c.get("processed", False),
                temperature=c.get("temperature", 0.0))
            rec["catalog_seqs"] = cat
            rec["final"] = [[b[0], b[1], b[2]] for b in beams]
        else:
            calls, outs = ref_shim.run_offline(
                reference_root, c["prompts"], beam_width=c["beam_width"], max_tokens=c["max_tokens"], vocab=c["vocab"],
                sigma=c["sigma"], seed=c["seed"], bf16=c.get("bf16", False), eos_token_id=c["eos"], ignore_eos=False,
                length_penalty=c["length_penalty"], processed=c.get("processed", False),
                temperature=c.get("temperature", 0.0))
            rec["final"] = [[[b[0], b[1], b[2]] for b in o] for o in outs]
        rec["calls"] = calls
        out.append(rec)
        print(c["name"], "steps", len(calls))
    with open(os.path.join(HERE, "reference_beams.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))


if __name__ == "__main__":
    main(sys.argv[1])
