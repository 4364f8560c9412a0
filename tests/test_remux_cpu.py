"""Logprobs remux on the CPU: the oracle against the reference's own outputs
(tests/golden/remux_cases.json, written by tests/golden/make_remux_golden.py)."""
import json
import os

import numpy as np
import pytest

from oracle import remux as orx

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "remux_cases.json")


def _cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


def _lps(rows):
    return np.array([[-np.inf if v == "-inf" else v for v in r] for r in rows], np.float32)


@pytest.mark.parametrize("idx", range(len(_cases())))
def test_oracle_matches_reference(idx):
    c = _cases()[idx]
    st, lps, ids, ranks = orx.remux(c["ws"], c["max_dim"], c["K"], np.array(c["lps"], np.float32),
                                    np.array(c["ids"], np.int32), np.array(c["ranks"], np.int32),
                                    np.array(c["st"], np.int32))
    np.testing.assert_array_equal(st, np.array(c["out_st"]))
    np.testing.assert_array_equal(lps, _lps(c["out_lps"]))
    np.testing.assert_array_equal(ids, np.array(c["out_ids"]))
    np.testing.assert_array_equal(ranks, np.array(c["out_ranks"]))
