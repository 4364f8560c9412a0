"""GPU parity at the geometry of every BASELINE configuration.

Each case keeps its configuration's beam width, vocabulary, logit dtype,
log-prob mode, catalog shape and step count, and cuts only the number of
requests (the oracle is a per-row NumPy loop):

  cfg1  fp32, 1 request, B = 128, 100k-item 3-level catalog (codebook 8192), 3 steps
  cfg2  bf16, B = 128, 1M-item catalog: test_parity_gpu.test_full_vocab_cfg2_rows
  cfg3  bf16, B = 512, 10M-item 4-level catalog (codebook 4096, Zipf 1.2), 4 steps
  cfg4  fp32, B = 256, unconstrained, processed log-probs with T = 0.7,
        repetition 1.2 and presence 0.5 over 64-token histories, 2 steps
  cfg5  vocab-sharded B = 1024: test_sharded_gpu.test_sharded_cfg5_true_geometry

Every case runs through both step kernels and checks both parity levels
(bit-exact given the device lse; reference arithmetic within 1e-5 fp32 /
2e-3 bf16) with the boundary near-ties counted and bounded.
"""
import numpy as np
import pytest

from helpers import Case, assert_step_parity, gpu_step, make_logits, next_inputs
from vllm_gr_ehaleva_b200.synthetic import CONFIGS, histories, initial_cum, make_catalog

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


@pytest.fixture(autouse=True, params=["auto", "stream"])
def step_kernel(request, monkeypatch):
    monkeypatch.setenv("GR_BEAM_KERNEL", request.param)
    return request.param


def _catalog(name):
    c = CONFIGS[name]
    return make_catalog(c["items"], c["levels"], c["codebook"], c["vocab"], c["zipf"], seed=1)


@pytest.fixture(scope="module")
def cfg3_catalog():
    return _catalog("cfg3")


def _constrained_chain(cfg_name, cat, R, seed):
    c = CONFIGS[cfg_name]
    B, V, dt = c["beams"], c["vocab"], c["dtype"]
    case = Case(logits32=make_logits(R, B, V, c["sigma"], seed, dt), dtype=dt, cum=initial_cum(R, B),
                node=np.full((R, B), cat.start_node, np.int32), beam_width=B, vocab_size=V, csr=cat.csr,
                hist=np.full((R, B, 1), cat.sid_begin, np.int32))
    for step in range(c["steps"]):
        gpu = gpu_step(case)
        assert_step_parity(case, gpu, label=f"{cfg_name} step {step}")
        # every new beam is a child of its parent's node
        for r in range(R):
            for i in range(B):
                p, t = gpu["sel_parent"][r, i], gpu["sel_token"][r, i]
                if p >= 0:
                    assert t in set(cat.csr.children(case.node[r, p]).tolist())
        case = next_inputs(case, gpu, make_logits(R, B, V, c["sigma"], seed + 1 + step, dt))
    return case


def test_cfg1_geometry():
    _constrained_chain("cfg1", _catalog("cfg1"), R=1, seed=0)


def test_cfg3_geometry(cfg3_catalog):
    _constrained_chain("cfg3", cfg3_catalog, R=1, seed=300)


def test_cfg4_geometry():
    c = CONFIGS["cfg4"]
    R, B, V, H = 1, c["beams"], c["vocab"], c["hist"]
    case = Case(logits32=make_logits(R, B, V, c["sigma"], 400, "f32"), dtype="f32", cum=initial_cum(R, B),
                node=np.full((R, B), -1, np.int32), beam_width=B, vocab_size=V,
                hist=histories(R, B, H, V, seed=3), mode="processed_logprobs",
                temperature=[c["temperature"]], rep=[c["rep"]], pres=[c["pres"]], freq=[c["freq"]])
    for step in range(2):
        gpu = gpu_step(case)
        assert_step_parity(case, gpu, label=f"cfg4 step {step}")
        nxt = next_inputs(case, gpu, make_logits(R, B, V, c["sigma"], 401 + step, "f32"))
        nxt.hist = case.hist      # the benchmark's fixed-length penalty history
        case = nxt


@pytest.mark.parametrize("dtype,mode", [("f32", "processed_logprobs"), ("bf16", "raw_logprobs")])
def test_streamed_rows_behind_the_request_bound(dtype, mode):
    # about 14 rows per SM: most rows start after their request already has a
    # bound, so in the selecting kernel the streaming warps take their
    # candidate pass, the finisher warp ends them, and (processed mode) the
    # penalised columns are masked through the per-row table
    R, B, V, H = 8, 256, 16384, 64
    proc = mode == "processed_logprobs"
    per_req = (lambda v: [v] * R) if proc else (lambda v: None)
    case = Case(logits32=make_logits(R, B, V, 3.0, 410, dtype), dtype=dtype, cum=initial_cum(R, B),
                node=np.full((R, B), -1, np.int32), beam_width=B, vocab_size=V,
                hist=histories(R, B, H, V, seed=5) if proc else None, mode=mode,
                temperature=per_req(0.7), rep=per_req(1.2), pres=per_req(0.5), freq=per_req(0.1))
    for step in range(2):
        gpu = gpu_step(case)
        assert_step_parity(case, gpu, label=f"many rows {dtype} step {step}")
        nxt = next_inputs(case, gpu, make_logits(R, B, V, 3.0, 411 + step, dtype))
        nxt.hist = case.hist      # a fixed penalty history (none in raw mode)
        case = nxt


def test_streamed_rows_whose_scores_rise_behind_the_bound():
    # beams are taken in order, and here every later beam scores far above the
    # bound its predecessors set: the survivors of a row that started with the
    # bound overflow its slot (they go on in the selectors' list) or that list
    # too (the row is read again exactly)
    R, B, V = 2, 256, 8192
    cum = np.tile(np.arange(B, dtype=np.float32), (R, 1)).astype(np.float32)
    case = Case(logits32=make_logits(R, B, V, 3.0, 420, "f32"), dtype="f32", cum=cum,
                node=np.full((R, B), -1, np.int32), beam_width=B, vocab_size=V)
    gpu = gpu_step(case)
    assert_step_parity(case, gpu, label="rising scores")
