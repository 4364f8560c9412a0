"""The worker hook's grouping of logit rows into step calls (host logic)."""
from types import SimpleNamespace

from vllm_gr_ehaleva_b200.engine import step_runs


def _s(b):
    return SimpleNamespace(beam_width=b)


def test_runs_group_consecutive_full_blocks_of_equal_width():
    sessions = {"a": _s(4), "b": _s(4), "c": _s(8), "d": _s(4), "e": _s(4)}
    cfg = [("a", 0, 4), ("b", 1, 4),          # one run of two sessions (rows 0..7)
           ("p", 2, 1),                       # a plain request's row splits runs
           ("d", 3, 4),                       # rows 9..12
           ("x", 4, 0),                       # a chunked prefill: no row, does not split
           ("e", 5, 4),                       # rows 13..16, joins d's run
           ("c", 6, 8),                       # other width: its own run (rows 17..24)
           ("a2", 7, 3)]                      # unregistered
    assert step_runs(cfg, sessions) == [(0, ["a", "b"], 4), (9, ["d", "e"], 4), (17, ["c"], 8)]


def test_partial_blocks_are_skipped():
    sessions = {"a": _s(4), "b": _s(4)}
    # a's block cut short by the chunk budget: not stepped; b still starts its own run at row 2
    assert step_runs([("a", 0, 2), ("b", 1, 4)], sessions) == [(2, ["b"], 4)]
    assert step_runs([], sessions) == []
