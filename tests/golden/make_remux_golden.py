"""Record the reference's logprobs remux as golden vectors.

    python tests/golden/make_remux_golden.py <reference checkout>

Runs the reference's own _remux_logprobs_tensors
(vllm_gr/v1/engine/engine_core_patch.py:383-445; torch code, here on CPU
tensors) on random sampler outputs for mixes of mega-decode requests (W
logit rows each), plain requests (one row) and chunked-prefill requests (no
row), and writes tests/golden/remux_cases.json with inputs and outputs.  The
fixture is committed; the tests read only it.
"""
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_shim  # noqa: E402


def main(reference_root):
    ref_shim.install_attention(reference_root)
    from vllm_gr.v1.engine.engine_core_patch import _remux_logprobs_tensors

    g = torch.Generator().manual_seed(4)
    cases = []
    for case in range(10):
        n = int(torch.randint(1, 7, (1,), generator=g))
        K = int(torch.randint(1, 9, (1,), generator=g))
        ws = [int(x) for x in torch.randint(0, 9, (n,), generator=g)]
        ws = [w if w != 2 else 1 for w in ws]       # plain requests give one row
        if case == 0:
            ws[0] = 0                               # a chunked prefill first
        rows = sum(ws)
        if rows == 0:
            ws[-1] = 3
            rows = 3
        lps = torch.randn(rows, K, generator=g)
        ids = torch.randint(0, 150000, (rows, K), generator=g, dtype=torch.int32)
        ranks = torch.randint(1, 1000, (rows,), generator=g, dtype=torch.int32)
        st = torch.randint(0, 150000, (rows, 1), generator=g, dtype=torch.int32)
        configs = [(f"r{i}", 0, w) for i, w in enumerate(ws)]
        max_dim = max(w * K for w in ws)
        o_st, o_lps, o_ids, o_ranks = _remux_logprobs_tensors(configs, max_dim, K, lps, ids, ranks, st)
        cases.append(dict(ws=ws, K=K, max_dim=max_dim, lps=lps.tolist(), ids=ids.tolist(), ranks=ranks.tolist(),
                          st=st.tolist(), out_st=o_st.tolist(),
                          out_lps=[[("-inf" if v == float("-inf") else v) for v in r] for r in o_lps.tolist()],
                          out_ids=o_ids.tolist(), out_ranks=o_ranks.tolist()))
    out = os.path.join(HERE, "remux_cases.json")
    with open(out, "w") as f:
        json.dump({"source": "vllm_gr/v1/engine/engine_core_patch.py:383-445 (reference _remux_logprobs_tensors)",
                   "cases": cases}, f, separators=(",", ":"))
    print(f"wrote {out}: {len(cases)} cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GR_REFERENCE_ROOT", ""))
