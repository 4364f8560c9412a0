"""GPU parity: the CUDA step against the CPU oracle (oracle/restated.py).

Two levels per case:
  * bit-exact: every output equal to the oracle run in device arithmetic with
    the GPU's own row log-sum-exp (isolates masking, scoring, selection order,
    tie-breaking, EOS handling, child nodes and the fork table);
  * reference arithmetic (float64 lse and score sums): candidate sets equal up
    to near-ties at the boundary, scores within 1e-5 relative (fp32 logits) or
    2e-3 (bf16 / fp16 logits), lse within 1e-5 relative.
"""
import numpy as np
import pytest

from helpers import (Case, assert_step_parity, gpu_step, make_logits, next_inputs, small_catalog,
                     tiny_catalog_csr)
from vllm_gr_ehaleva_b200.synthetic import histories, initial_cum

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=["auto", "stream"])
def step_kernel(request, monkeypatch):
    """Run every case through both step kernels: the automatic choice (the
    warp-specialised kernel where a step qualifies) and the streaming kernel."""
    monkeypatch.setenv("GR_BEAM_KERNEL", request.param)
    return request.param


def _constrained_case(dtype, R=3, NB=16, B=16, V=8192, seed=0, sigma=4.0, row_pad=0):
    cat = small_catalog(V=V)
    node = np.full((R, NB), cat.start_node, np.int32)
    return Case(logits32=make_logits(R, NB, V, sigma, seed, dtype), dtype=dtype, cum=initial_cum(R, NB),
                node=node, beam_width=B, vocab_size=V, csr=cat.csr,
                hist=np.full((R, NB, 1), cat.sid_begin, np.int32), row_pad=row_pad), cat


@pytest.mark.parametrize("dtype", ["bf16", "f32", "f16"])
def test_constrained_three_steps(dtype):
    case, cat = _constrained_case(dtype)
    for step in range(3):
        gpu = gpu_step(case)
        assert_step_parity(case, gpu)
        # every selected token is a child of its parent's node
        for r in range(case.R):
            for i in range(case.beam_width):
                p, t = gpu["sel_parent"][r, i], gpu["sel_token"][r, i]
                if p < 0:
                    continue
                assert t in set(cat.csr.children(case.node[r, p]).tolist())
        case = next_inputs(case, gpu, make_logits(case.R, case.NB, case.vocab_size, 4.0, 100 + step, dtype))


def test_constrained_first_step_single_beam():
    # the reference starts from one beam per request; B new beams come out of it
    cat = small_catalog()
    R, NB, B, V = 4, 1, 32, 8192
    case = Case(logits32=make_logits(R, NB, V, 4.0, 7, "bf16"), dtype="bf16", cum=np.zeros((R, NB), np.float32),
                node=np.full((R, NB), cat.start_node, np.int32), beam_width=B, vocab_size=V, csr=cat.csr)
    assert_step_parity(case, gpu_step(case))


def test_unaligned_row_stride():
    case, _ = _constrained_case("bf16", row_pad=3)
    assert_step_parity(case, gpu_step(case))
    case, _ = _constrained_case("f32", row_pad=1, seed=5)
    assert_step_parity(case, gpu_step(case))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_unconstrained_raw(dtype):
    R, NB, B, V = 3, 8, 16, 12000
    case = Case(logits32=make_logits(R, NB, V, 3.0, 11, dtype), dtype=dtype, cum=initial_cum(R, NB),
                node=np.full((R, NB), -1, np.int32), beam_width=B, vocab_size=V, eos=17)
    gpu = gpu_step(case)
    assert_step_parity(case, gpu)
    assert np.isfinite(gpu["eos_score"]).all()


def test_unconstrained_processed_penalties():
    R, NB, B, V, H = 3, 8, 16, 9000, 64
    case = Case(logits32=make_logits(R, NB, V, 3.0, 12, "f32"), dtype="f32", cum=initial_cum(R, NB),
                node=np.full((R, NB), -1, np.int32), beam_width=B, vocab_size=V,
                hist=histories(R, NB, H, V, seed=3), mode="processed_logprobs",
                temperature=[0.7, 1.0, 0.0], rep=[1.2, 1.5, 1.2], pres=[0.5, 0.0, 0.25], freq=[0.0, 0.2, 0.1])
    # make some penalised tokens the row's best so the penalty path decides the top
    x = case.logits32.copy()
    for r in range(R):
        for b in range(NB):
            x[r, b, case.hist[r, b, :4]] = 12.0 + b
    case.logits32 = x
    assert_step_parity(case, gpu_step(case))


def test_constrained_processed_penalties():
    case, cat = _constrained_case("f32", R=2, NB=8, B=8)
    case.mode = "processed_logprobs"
    case.temperature, case.rep, case.pres, case.freq = [0.7, 1.3], [1.2, 1.1], [0.5, 0.0], [0.0, 0.3]
    # history mentions level-1 tokens so children are penalised
    kids = cat.csr.children(cat.start_node)
    rng = np.random.default_rng(4)
    case.hist = rng.choice(kids, size=(2, 8, 32)).astype(np.int32)
    assert_step_parity(case, gpu_step(case))


@pytest.mark.parametrize("mode", ["raw_logprobs", "processed_logprobs"])
def test_reference_literal_mode(mode):
    # per_beam_k = B: each beam's own top-K of the full vocab, then catalog mask
    V = 4096
    cat = small_catalog(V=V, C=256, items=5000)
    R, NB, B = 2, 8, 8
    x = make_logits(R, NB, V, 4.0, 21, "f32")
    kids = cat.csr.children(cat.start_node)
    x[:, :, kids[:40]] += 9.0          # some allowed tokens reach the raw top-K
    case = Case(logits32=x, dtype="f32", cum=initial_cum(R, NB), node=np.full((R, NB), cat.start_node, np.int32),
                beam_width=B, vocab_size=V, csr=cat.csr, per_beam_k=B, mode=mode)
    gpu = gpu_step(case)
    assert_step_parity(case, gpu)


def test_reference_literal_sampled_dedup():
    # raw log-probs with penalties: the greedy (penalised) token can fall outside
    # the raw top-K and then replaces its K-th entry (vllm_gr/logprobs.py:47-52)
    V = 2048
    R, NB, B = 2, 4, 4
    x = make_logits(R, NB, V, 2.0, 31, "f32")
    hist = np.zeros((R, NB, 8), np.int32)
    for r in range(R):
        for b in range(NB):
            top = np.argsort(-x[r, b])[:8]
            hist[r, b] = top                       # penalise the whole raw top-8
    case = Case(logits32=x, dtype="f32", cum=initial_cum(R, NB), node=np.full((R, NB), -1, np.int32),
                beam_width=B, vocab_size=V, per_beam_k=B, hist=hist, rep=[3.0, 2.0], pres=[1.0, 1.0])
    assert_step_parity(case, gpu_step(case))


def test_eos_child_and_dead_and_padding():
    # catalog with an EOS child, a dead beam and fewer candidates than 2B
    V, eos = 64, 5
    csr = tiny_catalog_csr([[1, 2, 3], [1, 2, 4], [1, eos], [7, 8]])
    start = csr.walk([1])
    R, NB, B = 2, 3, 4
    x = make_logits(R, NB, V, 2.0, 41, "f32")
    node = np.array([[start, csr.walk([1, 2]), -2], [start, start, csr.walk([7])]], np.int32)
    case = Case(logits32=x, dtype="f32", cum=np.array([[-1, -2, -3], [-0.5, -0.7, -4]], np.float32),
                node=node, beam_width=B, vocab_size=V, csr=csr, eos=eos,
                hist=np.arange(R * NB * 2, dtype=np.int32).reshape(R, NB, 2))
    gpu = gpu_step(case)
    assert_step_parity(case, gpu)
    assert np.isfinite(gpu["eos_score"][0, 0]) and np.isnan(gpu["eos_score"][0, 1])
    assert (gpu["cand_parent"][0] == -1).any()        # padding present


def test_vocab_local_offset():
    # a column slice of the vocabulary (one shard's view) with global token ids
    case, cat = _constrained_case("bf16", R=2, NB=8, B=8)
    full = case.logits32
    off, VL = 4096, 4096
    case.logits32 = np.ascontiguousarray(full[:, :, off:off + VL])
    case.vocab_offset = off
    assert_step_parity(case, gpu_step(case))


def test_unconstrained_processed_column_slice():
    # unconstrained processed rows on a column slice of the vocabulary: the
    # penalty table keeps only the history tokens the slice holds
    R, NB, B, V, H = 2, 8, 8, 12000, 32
    off, VL = 5000, 4000
    full = make_logits(R, NB, V, 3.0, 14, "f32")
    hist = histories(R, NB, H, V, seed=6)
    hist[:, :, :8] = off + 7 + np.arange(8, dtype=np.int32)   # some history inside the slice for sure
    case = Case(logits32=np.ascontiguousarray(full[:, :, off:off + VL]), dtype="f32", cum=initial_cum(R, NB),
                node=np.full((R, NB), -1, np.int32), beam_width=B, vocab_size=V, vocab_offset=off,
                hist=hist, mode="processed_logprobs", temperature=[0.7, 1.3], rep=[1.2, 1.5], pres=[0.5, 0.1],
                freq=[0.1, 0.0])
    assert_step_parity(case, gpu_step(case))


@pytest.mark.slow
def test_full_vocab_cfg2_rows():
    # BASELINE cfg2 geometry (V=152064, B=128, bf16, 3-level codebook 8192) on 2 requests
    from vllm_gr_ehaleva_b200.synthetic import make_catalog
    cat = make_catalog(200_000, 3, 8192, 152064, 1.1, seed=1)
    R, NB, B, V = 2, 128, 128, 152064
    case = Case(logits32=make_logits(R, NB, V, 4.0, 0, "bf16"), dtype="bf16", cum=initial_cum(R, NB),
                node=np.full((R, NB), cat.start_node, np.int32), beam_width=B, vocab_size=V, csr=cat.csr,
                hist=np.full((R, NB, 1), cat.sid_begin, np.int32))
    for step in range(3):
        gpu = gpu_step(case)
        assert_step_parity(case, gpu)
        case = next_inputs(case, gpu, make_logits(R, NB, V, 4.0, 50 + step, "bf16"))


def test_mixed_rows_many_per_cta():
    # several rows per CTA (the warp-specialised kernel's two row slots cycle),
    # constrained rows at two catalog depths, rows without a node (re-read by
    # the row-end warps) and dead rows in one step
    cat = small_catalog(V=32768)
    R, NB, B, V = 8, 128, 32, 32768
    rng = np.random.default_rng(12)
    kinds = rng.integers(0, 10, size=(R, NB))
    first = cat.csr.child_node[cat.csr.row_ptr[cat.start_node]:cat.csr.row_ptr[cat.start_node + 1]]
    node = np.full((R, NB), cat.start_node, np.int32)
    deep = kinds >= 7
    node[deep] = first[rng.integers(0, len(first), size=int(deep.sum()))]   # one level down
    node[kinds == 0] = -1                      # unconstrained
    node[kinds == 1] = -2                      # dead
    case = Case(logits32=make_logits(R, NB, V, 4.0, 77, "bf16"), dtype="bf16", cum=initial_cum(R, NB),
                node=node, beam_width=B, vocab_size=V, csr=cat.csr)
    assert_step_parity(case, gpu_step(case))


def test_wide_beam_1024():
    # B = 1024 (cfg5's beam width): 2B = 2048 candidates per request; a few rows
    # without a node take the streamed path with its shorter sub-batches
    cat = small_catalog()
    R, NB, B, V = 1, 1024, 1024, 8192
    node = np.full((R, NB), cat.start_node, np.int32)
    node[0, 7] = -1
    node[0, 600] = -1
    case = Case(logits32=make_logits(R, NB, V, 4.0, 91, "bf16"), dtype="bf16", cum=initial_cum(R, NB), node=node,
                beam_width=B, vocab_size=V, csr=cat.csr)
    assert_step_parity(case, gpu_step(case))


def test_wide_beam_512_three_steps():
    # cfg3's beam width (2B = 1024: the request score histogram raises the bound)
    cat = small_catalog()
    R, NB, B, V = 2, 512, 512, 8192
    case = Case(logits32=make_logits(R, NB, V, 4.0, 92, "bf16"), dtype="bf16", cum=initial_cum(R, NB),
                node=np.full((R, NB), cat.start_node, np.int32), beam_width=B, vocab_size=V, csr=cat.csr,
                hist=np.full((R, NB, 1), cat.sid_begin, np.int32))
    for step in range(3):
        gpu = gpu_step(case)
        assert_step_parity(case, gpu)
        case = next_inputs(case, gpu, make_logits(R, NB, V, 4.0, 93 + step, "bf16"))


@pytest.mark.parametrize("dtype,mode", [("f32", "processed_logprobs"), ("bf16", "raw_logprobs")])
def test_unconstrained_full_vocab_many_rows(dtype, mode):
    # cfg4's geometry (V=152064, 64 penalised history tokens per beam) on 2
    # requests of 48 beams: later rows of a request filter their stream against
    # the request bound published by earlier rows; two steps
    R, NB, B, V, H = 2, 48, 48, 152064, 64
    sigma = 3.0
    kw = {}
    if mode == "processed_logprobs":
        kw = dict(temperature=[0.7, 0.7], rep=[1.2, 1.2], pres=[0.5, 0.5], freq=[0.0, 0.0])
    case = Case(logits32=make_logits(R, NB, V, sigma, 31, dtype), dtype=dtype, cum=initial_cum(R, NB),
                node=np.full((R, NB), -1, np.int32), beam_width=B, vocab_size=V,
                hist=histories(R, NB, H, V, seed=5), mode=mode, **kw)
    for step in range(2):
        gpu = gpu_step(case)
        assert_step_parity(case, gpu)
        nxt = next_inputs(case, gpu, make_logits(R, NB, V, sigma, 60 + step, dtype))
        nxt.hist = case.hist     # fixed-length penalty history, as in the benchmark
        case = nxt
