"""The reference's mega-request step message, restated (TEST INFRASTRUCTURE).

Only tests/ and bench.py's baseline leg use this: it rebuilds, for size and
time comparisons, the message the reference sends each decode step
(MegaRequestStepUpdate, vllm_gr/v1/engine/types.py:48-71) the way
serving_engine.py:108-142 fills it, and the engine core's token list from it
(vllm_gr/v1/engine/core.py:109-112).  SamplingParams is carried as the same
pre-encoded bytes as in vllm_gr_ehaleva_b200.wire, so the comparison covers the
beam content only.
"""
from __future__ import annotations

import msgspec


class RefStepUpdate(msgspec.Struct, array_like=True, omit_defaults=True, gc=False):
    session_id: str
    parent_beam_ids: list[str]
    child_beam_ids: list[str]
    beam_tokens: list[list[int]]
    pruned_ids: list[str]
    prefix_len: int
    beam_width: int
    sampling_params: bytes = b""
    eos_token_id: int | None = None


def build(session_id, fork_info, prev_ids, beams_tokens, batch, prefix_len, eos_token_id=None, params=b""):
    """fork_info: [(parent index, token)] per new beam; beams_tokens: each new
    beam's full token list (prompt included)."""
    parent_ids, child_ids, beam_tokens = [], [], []
    for new_idx, (p, _tok) in enumerate(fork_info):
        parent_ids.append(prev_ids[p])
        child_ids.append(f"{batch}-beam-{new_idx}")
        beam_tokens.append(beams_tokens[new_idx][prefix_len:])
    used = set(parent_ids)
    pruned = [pid for pid in prev_ids if pid not in used]
    return RefStepUpdate(session_id=session_id, parent_beam_ids=parent_ids, child_beam_ids=child_ids,
                         beam_tokens=beam_tokens, pruned_ids=pruned, prefix_len=prefix_len,
                         beam_width=len(fork_info), sampling_params=params, eos_token_id=eos_token_id)


def mega_token_ids(update, prefill_tokens):
    out = list(prefill_tokens)
    for t in update.beam_tokens:
        out.extend(t)
    return out
