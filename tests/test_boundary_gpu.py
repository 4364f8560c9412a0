"""Streamed rows whose kept top-k boundary meets equal values.

A streamed row (no catalog node, or the reference-literal per-beam top-K)
keeps only its best keys by value once its list fills up.  Dropping columns is
exact unless a dropped column can score as high as the row's selection
boundary: distinct values can round to one float32 score (cum + (y - lse)) or
log-prob (y - lse).  These cases build exactly that, and the step must still
give the oracle's selection bit for bit (it re-reads such a row exactly):

  * bf16: hundreds of logits equal to the boundary value (equal values keep
    their flat-index order; no re-read is needed, no error may be raised);
  * fp32: a cluster of distinct values whose scores collapse onto one or two
    float32 values next to a large cumulative score (the re-read decides by
    flat index);
  * fp32, reference-literal top-K: the same collapse in the log-prob domain
    (checked bit for bit in the device's arithmetic: the per-beam top-K
    boundary itself lies inside the cluster there).
"""
import numpy as np
import pytest

from helpers import Case, assert_bit_exact, assert_step_parity, gpu_step, oracle_step, round_to

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=["auto", "stream", "ws"])
def step_kernel(request, monkeypatch):
    monkeypatch.setenv("GR_BEAM_KERNEL", request.param)
    return request.param


def test_bf16_many_equal_values_at_the_boundary():
    R, NB, B, V = 2, 4, 16, 8192
    rng = np.random.default_rng(51)
    x = rng.standard_normal((R, NB, V), dtype=np.float32)
    for r in range(R):
        for b in range(NB):
            cols = rng.choice(V, 310, replace=False)
            x[r, b, cols[:300]] = 5.0            # 2B and 2B + slack fall inside this run of equal values
            x[r, b, cols[300:]] = 6.0
    x = round_to(x, "bf16")
    cum = np.array([[-1.0, -1.5, -2.0, -3.0], [-0.5, -0.5, -4.0, -9.0]], np.float32)
    case = Case(logits32=x, dtype="bf16", cum=cum, node=np.full((R, NB), -1, np.int32), beam_width=B,
                vocab_size=V)
    assert_step_parity(case, gpu_step(case))


def test_f32_scores_collapse_next_to_a_large_cumulative_score():
    R, NB, B, V = 1, 4, 16, 8192
    rng = np.random.default_rng(52)
    x = (rng.standard_normal((R, NB, V), dtype=np.float32) * 0.5).astype(np.float32)
    for b in range(NB):
        cols = rng.choice(V, 300, replace=False)
        # distinct values 1e-6 apart: one float32 ulp of -5006 spans all of them
        x[0, b, cols] = (np.float32(5.0) + rng.permutation(300).astype(np.float32) * np.float32(1e-6))
    cum = np.array([[-5000.0, -5000.5, -5001.0, -5002.0]], np.float32)
    case = Case(logits32=x, dtype="f32", cum=cum, node=np.full((R, NB), -1, np.int32), beam_width=B, vocab_size=V)
    # reference arithmetic (float64 sums) separates what float32 ties: the
    # sets may differ anywhere in the collapsed cluster, within tolerance
    assert_step_parity(case, gpu_step(case), max_near_ties=4 * B)


def test_literal_top_k_log_probs_collapse():
    R, NB, B, V = 1, 2, 8, 4096
    rng = np.random.default_rng(53)
    x = (np.float32(-20.0) + rng.standard_normal((R, NB, V), dtype=np.float32) * 0.1).astype(np.float32)
    for b in range(NB):
        cols = rng.choice(V, 300, replace=False)
        # values one float32 ulp of 0.5 apart; their log-probs (about -5.7) share ulps by the eight
        x[0, b, cols] = (np.float32(0.5) + rng.permutation(300).astype(np.float32) * np.float32(6e-8))
    case = Case(logits32=x, dtype="f32", cum=np.array([[-1.0, -1.25]], np.float32),
                node=np.full((R, NB), -1, np.int32), beam_width=B, vocab_size=V, per_beam_k=B)
    gpu = gpu_step(case)
    assert gpu["err"] == 0
    # Here each beam's own top-K boundary lies inside the collapsed cluster, so
    # float64 arithmetic would pick other members of it: the check is the
    # bit-exact one in the device's float32 arithmetic, given its lse.
    assert_bit_exact(gpu, oracle_step(case, arith="device", lse_override=gpu["lse"]))
    ref = oracle_step(case, arith="reference")
    assert np.allclose(gpu["lse"], ref["lse"], rtol=1e-5, atol=0)
