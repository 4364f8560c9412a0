"""The CUDA step against the reference's own beam-search loops (golden vectors).

Same fixtures as tests/test_golden_reference.py, but the package's beam loop
is driven by the device step: the beams requested at every step, the final
sequences and finish reasons must equal the reference's, cumulative log-probs
within 1e-5 relative (fp32 logits) or 2e-3 (bf16 logits, which the step reads
as bf16).  Processed-mode cases run the step in processed mode with the
temperature the reference's loop passed.
"""
import pytest

from test_golden_reference import CASES, recorder, same_final, step_mode, tolerance
from vllm_gr_ehaleva_b200.beam_search import beam_search, device_step_fn
from vllm_gr_ehaleva_b200.catalog import csr_from_sequences

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_device_matches_reference_loops(case):
    calls = []
    mode, temp = step_mode(case)
    kw = dict(dtype="bf16" if case.get("bf16") else "f32", logprobs_mode=mode, temperature=temp)
    if case["kind"] == "online":
        csr = csr_from_sequences(case["catalog_seqs"])
        cat = case["catalog"]
        res = beam_search([case["prompt"]], recorder(case, calls), beam_width=case["beam_width"],
                          max_tokens=case["max_tokens"], vocab_size=case["vocab"],
                          step_fn=device_step_fn(csr=csr, **kw), catalog=csr, begin_token=cat["begin"],
                          end_token=cat["end"], eos_token_id=case["eos"], online=True)
        same_final(res[0], case["final"], tolerance(case))
    else:
        res = beam_search(case["prompts"], recorder(case, calls), beam_width=case["beam_width"],
                          max_tokens=case["max_tokens"], vocab_size=case["vocab"],
                          step_fn=device_step_fn(per_beam_k=case["beam_width"], **kw), eos_token_id=case["eos"],
                          online=False, length_penalty=case["length_penalty"])
        for got, ref in zip(res, case["final"]):
            same_final(got, ref, tolerance(case))
    assert len(calls) == len(case["calls"])
    for mine, theirs in zip(calls, case["calls"]):
        assert sorted(map(tuple, mine)) == sorted(map(tuple, theirs))
