"""Record the reference's mega-request step updates as golden vectors.

    python tests/golden/make_wire_golden.py <reference checkout>

Calls the reference's own `_mega_request_step`
(vllm_gr/entrypoints/openai/serving_engine.py:91-168) on a mock engine client
that captures the MegaRequestStepUpdate it sends (types.py:48-71), for random
forks of random beams (catalog-like token ids, several beam widths and step
counts, beams that fork into several children and parents that are pruned),
and writes tests/golden/wire_updates.json: per case the inputs (fork_info,
the previous step's beam ids, the new beams' token lists, prefix length, batch
id) and the fields of the captured message.  The fixture is committed; the
tests read only it.
"""
import asyncio
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_shim  # noqa: E402


class _Out:
    finished = True


class _MockClient:
    def __init__(self):
        self.updates = []

    def register_beam_output(self, session_id, tokens, params, **kw):
        q = asyncio.Queue()
        q.put_nowait(_Out())
        return q

    async def mega_request_step_update(self, update):
        self.updates.append(update)


def main(reference_root):
    ref_shim.install(reference_root)
    from vllm.sampling_params import SamplingParams

    import vllm_gr.entrypoints.openai.serving_engine as se

    class Beam:
        def __init__(self, tokens):
            self.tokens = tokens

    rng = np.random.default_rng(11)
    cases = []
    for case in range(12):
        prev_w = int(rng.choice([1, 4, 16, 128]))
        w = int(rng.choice([4, 16, 128]))
        prefix_len = int(rng.integers(3, 40))
        steps = int(rng.integers(1, 6))
        prompt = rng.integers(0, 150000, prefix_len).tolist()
        prev_batch = f"req{case}-{rng.integers(1 << 30):08x}"
        batch = f"req{case}-{rng.integers(1 << 30):08x}"
        prev_ids = [f"{prev_batch}-beam-{i}" for i in range(prev_w)]
        parents = rng.integers(0, prev_w, w)
        parents[: min(w, 2)] = parents[0]                      # one parent forking into several children
        gen = rng.integers(127488, 152064, (w, steps))         # SID-range tokens
        beams = [Beam(prompt + gen[i].tolist()) for i in range(w)]
        fork_info = [(int(parents[i]), int(gen[i, -1])) for i in range(w)]
        client = _MockClient()
        asyncio.run(se._mega_request_step(client, session_id=f"sess{case}", fork_info=fork_info,
                                          prev_beam_internal_ids=prev_ids, all_beams=beams,
                                          request_id_batch=batch, beam_search_params=SamplingParams(n=1),
                                          eos_token_id=151643, lora_request=None, trace_headers=None,
                                          prefix_len=prefix_len, priority=0, data_parallel_rank=None))
        u = client.updates[0]
        cases.append(dict(
            inputs=dict(session_id=f"sess{case}", prev_batch=prev_batch, prev_width=prev_w, batch=batch,
                        prefix_len=prefix_len, parents=parents.tolist(), tokens=gen.tolist(), eos_token_id=151643),
            update=dict(session_id=u.session_id, parent_beam_ids=list(u.parent_beam_ids),
                        child_beam_ids=list(u.child_beam_ids), beam_tokens=[list(t) for t in u.beam_tokens],
                        pruned_ids=list(u.pruned_ids), prefix_len=u.prefix_len, beam_width=u.beam_width,
                        eos_token_id=u.eos_token_id)))
    out = os.path.join(HERE, "wire_updates.json")
    with open(out, "w") as f:
        json.dump({"source": "vllm_gr/entrypoints/openai/serving_engine.py:91-168 (reference _mega_request_step)",
                   "cases": cases}, f, separators=(",", ":"))
    print(f"wrote {out}: {len(cases)} cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GR_REFERENCE_ROOT", ""))
