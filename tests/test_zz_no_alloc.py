"""gr_beam_step_noalloc: the step for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc themselves — code that runs
where an allocation would synchronise the device or bypass the process's memory
pool, or a host without an allocator of its own — so they cannot hand
gr_beam_step a workspace.  gr_beam_step_noalloc runs the same step on a fixed
scratch array the library keeps in device memory.  These tests call it through
the C ABI and check that calls in a row give, bit for bit, what the workspace
entry point gives on the same inputs (and, once, what the oracle gives), and
that a request larger than the built-in scratch is refused.  (This file is named to be collected last.)
"""
import ctypes

import numpy as np
import pytest

from helpers import Case, make_logits, small_catalog, to_device_logits
from vllm_gr_ehaleva_b200.synthetic import initial_cum

pytestmark = pytest.mark.gpu

KEYS = ("cand_score", "cand_token", "cand_parent", "sel_score", "sel_token", "sel_parent", "sel_node",
        "eos_score", "hist_out", "lse")


def _run_noalloc(case: Case, device="cuda"):
    """Call gr_beam_step_noalloc through ctypes with freshly allocated outputs."""
    import torch
    from vllm_gr_ehaleva_b200 import _lib
    from vllm_gr_ehaleva_b200.sample.beam_search_sampler import _DTYPES, _ptr, make_desc

    lib = _lib.load()
    logits = to_device_logits(case, device)
    R, NB = case.cum.shape
    VL = logits.shape[-1]
    B = case.beam_width
    T = 0 if case.hist is None else case.hist.shape[2]
    csr = [torch.from_numpy(a).to(device) for a in (case.csr.row_ptr, case.csr.child_tok, case.csr.child_node)]
    cum = torch.from_numpy(case.cum).to(device)
    node = torch.from_numpy(case.node).to(device)
    hist = None if case.hist is None else torch.from_numpy(case.hist).to(device)
    f32 = dict(dtype=torch.float32, device=device)
    i32 = dict(dtype=torch.int32, device=device)
    out = {"cand_score": torch.empty((R, 2 * B), **f32), "cand_token": torch.empty((R, 2 * B), **i32),
           "cand_parent": torch.empty((R, 2 * B), **i32), "sel_score": torch.empty((R, B), **f32),
           "sel_token": torch.empty((R, B), **i32), "sel_parent": torch.empty((R, B), **i32),
           "sel_node": torch.empty((R, B), **i32), "eos_score": torch.empty((R, NB), **f32),
           "hist_out": torch.empty((R, B, T + 1), **i32), "lse": torch.empty((R, NB), **f32),
           "err": torch.zeros(1, **i32)}
    desc = make_desc(R=R, NB=NB, B=B, V=case.vocab_size, VL=VL, voff=case.vocab_offset,
                     row_stride=logits.stride(0), dtype=_DTYPES[logits.dtype], mode=0, K=0, eos=-1, T=T,
                     N=int(csr[0].numel()) - 1, E=int(csr[1].numel()))
    io = _lib.StepIO()
    io.logits, io.cum, io.node = _ptr(logits), _ptr(cum), _ptr(node)
    io.row_ptr, io.child_tok, io.child_node = _ptr(csr[0]), _ptr(csr[1]), _ptr(csr[2])
    io.hist_in = _ptr(hist)
    for k, t in out.items():
        setattr(io, "err" if k == "err" else k, _ptr(t))
    stream = torch.cuda.current_stream(device)
    status = lib.gr_beam_step_noalloc(ctypes.byref(desc), ctypes.byref(io), ctypes.c_void_p(stream.cuda_stream))
    torch.cuda.synchronize()
    res = {k: v.cpu().numpy() for k, v in out.items() if k != "err"}
    res["err"] = int(out["err"].item())
    return status, res


def _case(seed, R=3, B=16):
    cat = small_catalog()
    NB, V = B, 8192
    return Case(logits32=make_logits(R, NB, V, 4.0, seed, "bf16"), dtype="bf16", cum=initial_cum(R, NB),
                node=np.full((R, NB), cat.start_node, np.int32), beam_width=B, vocab_size=V, csr=cat.csr,
                hist=np.full((R, NB, 1), cat.sid_begin, np.int32))


def _same(a, b):
    """Bit for bit: the same kernels ran on the same inputs, only the scratch
    differs (NaN equals NaN)."""
    for k in KEYS:
        x, y = np.asarray(a[k]), np.asarray(b[k])
        assert x.shape == y.shape, k
        if x.dtype.kind == "f":
            same = (x.view(np.uint32) == y.view(np.uint32)) | (np.isnan(x) & np.isnan(y))
            assert same.all(), k
        else:
            assert np.array_equal(x, y), k


def test_noalloc_matches_workspace_entry_point_twice():
    from helpers import gpu_step
    for seed in (101, 202):                      # two calls in a row share the scratch array
        case = _case(seed)
        ref = gpu_step(case)                     # gr_beam_step with a caller workspace
        status, got = _run_noalloc(case)
        assert status == 0, f"gr_beam_step_noalloc returned {status}"
        assert got["err"] == 0 and ref["err"] == 0
        _same(got, ref)


def test_noalloc_large_small_large():
    # B = 256 (2B = 512): the per-request score histogram, the largest part of
    # the scratch a step must clear, lives in the shared array too.  A large
    # call, a small one, then the large one again: leftover histogram bins or
    # list counts from an earlier call would show as a difference.
    from helpers import assert_step_parity, gpu_step
    large, small = _case(303, R=4, B=256), _case(404, R=2, B=16)
    for i, case in enumerate((large, small, large)):
        ref = gpu_step(case)
        status, got = _run_noalloc(case)
        assert status == 0, f"gr_beam_step_noalloc returned {status}"
        assert got["err"] == 0 and ref["err"] == 0
        _same(got, ref)
        if i == 0:
            assert_step_parity(case, got)        # and against the oracle directly


def test_noalloc_rejects_requests_beyond_its_scratch():
    from vllm_gr_ehaleva_b200 import _lib
    from vllm_gr_ehaleva_b200.sample.beam_search_sampler import make_desc
    lib = _lib.load()
    # 512 requests x 512 beams x 2B=1024 slots x 8 bytes is far beyond the built-in scratch
    desc = make_desc(R=512, NB=512, B=512, V=152064, VL=152064, voff=0, row_stride=152064, dtype=1, mode=0,
                     K=0, eos=-1, T=0, N=0, E=0)
    need = ctypes.c_size_t(0)
    assert lib.gr_beam_step_workspace_size(ctypes.byref(desc), ctypes.byref(need)) == 0
    assert need.value > _lib.NOALLOC_SCRATCH_BYTES
    io = _lib.StepIO()
    assert lib.gr_beam_step_noalloc(ctypes.byref(desc), ctypes.byref(io), None) == -5   # GR_ERR_WORKSPACE
