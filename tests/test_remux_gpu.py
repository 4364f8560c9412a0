"""GPU parity of gr_remux_logprobs: bit-exact against the reference's own
outputs (golden) and against the oracle on larger mixes and other dtypes."""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from oracle import remux as orx  # noqa: E402
from vllm_gr_ehaleva_b200.engine import remux_logprobs_tensors  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "remux_cases.json")
DEV = "cuda"


def _cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


def test_matches_reference_outputs():
    for c in _cases():
        cfg = [(f"r{i}", 0, w) for i, w in enumerate(c["ws"])]
        lps = torch.tensor(c["lps"], dtype=torch.float32, device=DEV)
        ids = torch.tensor(c["ids"], dtype=torch.int32, device=DEV)
        ranks = torch.tensor(c["ranks"], dtype=torch.int32, device=DEV)
        st = torch.tensor(c["st"], dtype=torch.int32, device=DEV)
        o_st, o_lps, o_ids, o_ranks = remux_logprobs_tensors(cfg, c["max_dim"], c["K"], lps, ids, ranks, st)
        exp_lps = np.array([[-np.inf if v == "-inf" else v for v in r] for r in c["out_lps"]], np.float32)
        np.testing.assert_array_equal(o_lps.cpu().numpy(), exp_lps)
        assert o_st.cpu().tolist() == c["out_st"] and o_ids.cpu().tolist() == c["out_ids"]
        assert o_ranks.cpu().tolist() == c["out_ranks"]


@pytest.mark.parametrize("int_dtype", [torch.int32, torch.int64])
def test_large_mix_and_optional_arrays(int_dtype):
    rng = np.random.default_rng(2)
    ws = rng.choice([0, 1, 128, 129, 64], 300).tolist()
    K = 129
    rows = sum(ws) + 5
    lps = torch.randn(rows, K + 3, device=DEV)                        # wider than K: a column slice
    ids = torch.randint(0, 150000, (rows, K + 3), device=DEV, dtype=int_dtype)
    ranks = torch.randint(1, 99, (rows,), device=DEV, dtype=int_dtype)
    st = torch.randint(0, 150000, (rows, 1), device=DEV, dtype=int_dtype)
    cfg = [(i, 0, w) for i, w in enumerate(ws)]
    max_dim = max(w * K for w in ws)
    o = remux_logprobs_tensors(cfg, max_dim, K, lps, ids, ranks, st)
    e = orx.remux(ws, max_dim, K, lps.cpu().numpy(), ids.cpu().numpy(), ranks.cpu().numpy(), st.cpu().numpy())
    for a, b in zip(o, e):
        np.testing.assert_array_equal(a.cpu().numpy(), b)
    o2 = remux_logprobs_tensors(cfg, max_dim, K, lps, None, None, st)
    assert o2[2] is None and o2[3] is None
    np.testing.assert_array_equal(o2[1].cpu().numpy(), e[1])
    # the reference's early return
    r = remux_logprobs_tensors(cfg, 0, K, lps, ids, ranks, st)
    assert r[0] is st and r[1] is lps
