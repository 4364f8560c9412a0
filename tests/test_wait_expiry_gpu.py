"""The bounded waits of the step kernels, made to run out.

Every mbarrier wait in the step kernels gives up after a fixed time limit,
sets GR_DEVERR_TIMEOUT in the caller's error word, drains the copies its CTA
has in flight and returns, so that a copy that never lands cannot hang the
GPU.  The test hook GR_TEST_STALL_COPIES=1 makes the producers issue no bulk
copies at all (nothing in flight; the consumers' first wait can only expire).
The call must come back within a few wait limits with the bit set, and the
next step on the same stream must be correct again.

Every step kernel runs a case: the warp-specialised ones decide to leave a
row on one value per role (taken between two barriers), so a wait that gives
up on some threads only cannot split the role at a barrier.
"""
import time

import numpy as np
import pytest

from helpers import Case, assert_step_parity, gpu_step, make_logits, small_catalog
from vllm_gr_ehaleva_b200.synthetic import initial_cum

pytestmark = pytest.mark.gpu

GR_DEVERR_TIMEOUT = 0x4


@pytest.mark.parametrize("kernel", ["auto", "stream"])
def test_bounded_wait_expiry_reports_timeout(kernel, monkeypatch):
    cat = small_catalog()
    R, NB, B, V = 2, 8, 8, 8192
    case = Case(logits32=make_logits(R, NB, V, 4.0, 71, "bf16"), dtype="bf16", cum=initial_cum(R, NB),
                node=np.full((R, NB), cat.start_node, np.int32), beam_width=B, vocab_size=V, csr=cat.csr,
                hist=np.full((R, NB, 1), cat.sid_begin, np.int32))
    monkeypatch.setenv("GR_BEAM_KERNEL", kernel)
    monkeypatch.setenv("GR_TEST_STALL_COPIES", "1")
    t0 = time.monotonic()
    stalled = gpu_step(case)
    elapsed = time.monotonic() - t0
    assert stalled["err"] & GR_DEVERR_TIMEOUT, f"error word {stalled['err']:#x}"
    assert elapsed < 30.0, f"the expired waits took {elapsed:.1f} s to return"
    monkeypatch.delenv("GR_TEST_STALL_COPIES")
    assert_step_parity(case, gpu_step(case))


def test_bounded_wait_expiry_streamed_rows(monkeypatch):
    # a step without a catalog (the selecting kernel: streamers, selectors,
    # producer and finisher all wait on one another)
    R, NB, B, V = 2, 8, 8, 8192
    case = Case(logits32=make_logits(R, NB, V, 3.0, 72, "f32"), dtype="f32", cum=initial_cum(R, NB),
                node=np.full((R, NB), -1, np.int32), beam_width=B, vocab_size=V)
    monkeypatch.setenv("GR_TEST_STALL_COPIES", "1")
    t0 = time.monotonic()
    stalled = gpu_step(case)
    elapsed = time.monotonic() - t0
    assert stalled["err"] & GR_DEVERR_TIMEOUT, f"error word {stalled['err']:#x}"
    assert elapsed < 30.0, f"the expired waits took {elapsed:.1f} s to return"
    monkeypatch.delenv("GR_TEST_STALL_COPIES")
    assert_step_parity(case, gpu_step(case))
