"""The int32 step message (vllm_gr_ehaleva_b200.wire) against the reference's
own step updates: golden messages recorded from serving_engine._mega_request_step
(tests/golden/make_wire_golden.py), the restated reference message, round trips."""
import json
import os

import numpy as np
import pytest

from oracle import wire_ref
from vllm_gr_ehaleva_b200 import wire

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "wire_updates.json")


def _cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("idx", range(len(_cases())))
def test_matches_reference_message(idx):
    c = _cases()[idx]
    i = c["inputs"]
    fork = wire.build_step_fork(i["session_id"], i["batch"], i["prev_batch"], i["prev_width"], i["parents"],
                                i["tokens"], i["prefix_len"], eos_token_id=i["eos_token_id"])
    got = wire.step_update_fields(wire.decode(wire.encode(fork)))
    assert got == c["update"]


@pytest.mark.parametrize("idx", range(len(_cases())))
def test_core_token_list_and_restated_reference(idx):
    c = _cases()[idx]
    i = c["inputs"]
    prefill = list(range(1000, 1000 + i["prefix_len"]))
    fork = wire.build_step_fork(i["session_id"], i["batch"], i["prev_batch"], i["prev_width"], i["parents"],
                                i["tokens"], i["prefix_len"], eos_token_id=i["eos_token_id"])
    prev_ids = [f"{i['prev_batch']}-beam-{j}" for j in range(i["prev_width"])]
    beams = [prefill + t for t in i["tokens"]]
    ref = wire_ref.build(i["session_id"], list(zip(i["parents"], [t[-1] for t in i["tokens"]])), prev_ids, beams,
                         i["batch"], i["prefix_len"], eos_token_id=i["eos_token_id"])
    assert ref.parent_beam_ids == c["update"]["parent_beam_ids"] and ref.pruned_ids == c["update"]["pruned_ids"]
    np.testing.assert_array_equal(wire.mega_token_ids(fork, prefill), wire_ref.mega_token_ids(ref, prefill))
    assert len(wire.encode(fork)) < len(__import__("msgspec").msgpack.encode(ref))


def test_rejects_bad_shapes_and_parents():
    with pytest.raises(ValueError):
        wire.build_step_fork("s", "b", "p", 4, [0, 1], [[1, 2, 3]], 5)        # 2 parents, 1 token row
    with pytest.raises(ValueError):
        wire.build_step_fork("s", "b", "p", 4, [0, 4], [[1], [2]], 5)          # parent 4 of 4 beams
    f = wire.build_step_fork("s", "b", "p", 1, np.zeros(0, np.int32), np.zeros((0, 3), np.int32), 5)
    assert wire.step_update_fields(f)["pruned_ids"] == ["p-beam-0"]


def test_params_travel_as_bytes():
    raw = b"\x81\xa1n\x01"
    f = wire.build_step_fork("s", "b", "p", 2, [1, 1], [[7], [8]], 3, sampling_params=raw)
    g = wire.decode(wire.encode(f))
    assert g.sampling_params == raw and wire.parents_of(g).tolist() == [1, 1]
