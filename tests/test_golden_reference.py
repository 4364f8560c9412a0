"""The oracle against the reference's own beam-search loops (golden vectors).

tests/golden/reference_beams.json was recorded by running the reference's
serving_engine.beam_search (catalog-constrained) and llm.beam_search
(unconstrained, EOS, length penalty) unmodified on a mock engine
(tests/golden/make_golden.py, oracle/ref_shim.py).  Here the package's beam
loop (vllm_gr_ehaleva_b200/beam_search.py) is driven by the oracle's step on
the same content-addressed logits (the offline loop in the reference-literal
mode, per_beam_k = beam width, which is what llm.py computes): every step must
request exactly the reference's beams, and the final sequences, finish reasons
and cumulative log-probs must match (1e-5 relative for float32 logits, 2e-3 for
bf16).  Cases with "processed" ran the mock engine in vLLM's processed_logprobs
mode with the temperature the reference's loop passed; the step runs in the
same mode with that temperature.
"""
import json
import os

import numpy as np
import pytest

from oracle import restated as O
from oracle.ref_shim import beam_logits
from vllm_gr_ehaleva_b200.beam_search import beam_search
from vllm_gr_ehaleva_b200.catalog import csr_from_sequences

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_beams.json")
with open(GOLDEN) as f:
    CASES = json.load(f)


def step_mode(case):
    """(logprobs mode, temperature) the case's engine ran with."""
    if case.get("processed"):
        return "processed_logprobs", float(case.get("temperature", 0.0))
    return "raw_logprobs", None


def tolerance(case):
    return 2e-3 if case.get("bf16") else 1e-5


def oracle_step_fn(csr, per_beam_k=0, case=None):
    ocsr = None if csr is None else O.CSR(csr.row_ptr, csr.child_tok, csr.child_node)
    mode, temp = step_mode(case or {})

    def step(logits32, cum, node, *, beam_width, vocab_size, eos_token_id):
        kw = {}
        if mode == "processed_logprobs":
            kw = dict(logprobs_mode=O.PROCESSED, temperature=[temp] * cum.shape[0])
        out = dict(O.beam_step(logits32, cum, node, ocsr, beam_width=beam_width, vocab_size=vocab_size,
                               eos_token_id=eos_token_id, per_beam_k=per_beam_k, arith="reference", **kw))
        out["sel_score"] = out["cand_score64"][:, :beam_width]
        return out
    return step


def recorder(case, calls):
    def logits_fn(rows):
        calls.append([list(r) for r in rows])
        return np.stack([beam_logits(r, case["vocab"], case["sigma"], case["seed"], case.get("bf16", False))
                         for r in rows])
    return logits_fn


def same_final(got, ref, tol=1e-5):
    assert len(got) == len(ref)
    for (gt, gc, gf), (rt, rc, rf) in zip(got, ref):
        assert list(gt) == list(rt)
        assert (gf or None) == (rf or None) or (gf == "length" and rf == "length")
        assert abs(gc - rc) <= tol * max(1.0, abs(rc)), (gc, rc)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_loops(case):
    calls = []
    if case["kind"] == "online":
        csr = csr_from_sequences(case["catalog_seqs"])
        cat = case["catalog"]
        res = beam_search([case["prompt"]], recorder(case, calls), beam_width=case["beam_width"],
                          max_tokens=case["max_tokens"], vocab_size=case["vocab"],
                          step_fn=oracle_step_fn(csr, case=case), catalog=csr, begin_token=cat["begin"],
                          end_token=cat["end"], eos_token_id=case["eos"], online=True)
        same_final(res[0], case["final"], tolerance(case))
    else:
        res = beam_search(case["prompts"], recorder(case, calls), beam_width=case["beam_width"],
                          max_tokens=case["max_tokens"], vocab_size=case["vocab"],
                          # llm.py takes each beam's own top-K (K = beam width) before the EOS
                          # filter: the reference-literal mode
                          step_fn=oracle_step_fn(None, per_beam_k=case["beam_width"], case=case),
                          eos_token_id=case["eos"], online=False, length_penalty=case["length_penalty"])
        for got, ref in zip(res, case["final"]):
            same_final(got, ref, tolerance(case))
    # every step asked the engine for the same beams (order free: the reference's is unspecified)
    assert len(calls) == len(case["calls"])
    for mine, theirs in zip(calls, case["calls"]):
        assert sorted(map(tuple, mine)) == sorted(map(tuple, theirs))
