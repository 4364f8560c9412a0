"""The caller's device error word with and without GR_STEP_CLEAR_ERR.

With the flag the step zeroes the word itself before any kernel reports into
it (beam_step uses this, so no fill kernel runs per step); a bad node id found
by the row metadata kernel is then reported by the merge kernel.  Without it
the step ORs its bits into the word as it stands.
"""
import ctypes

import numpy as np
import pytest

from helpers import OUT_KEYS, Case, assert_bit_exact, make_logits, small_catalog, to_device_logits
from vllm_gr_ehaleva_b200.synthetic import initial_cum

pytestmark = pytest.mark.gpu

GR_DEVERR_BAD_NODE = 0x1


def _call(case, cat, node, err_fill, clear):
    import torch
    from vllm_gr_ehaleva_b200 import _lib
    from vllm_gr_ehaleva_b200.sample.beam_search_sampler import _prepare
    dev = torch.device("cuda")
    csr = tuple(torch.from_numpy(a).to(dev) for a in (cat.csr.row_ptr, cat.csr.child_tok, cat.csr.child_node))
    desc, io, out, ws, s, _keep = _prepare(
        to_device_logits(case, dev), torch.from_numpy(case.cum).to(dev), torch.from_numpy(node).to(dev),
        beam_width=case.beam_width, csr=csr, vocab_size=case.vocab_size,
        hist=torch.from_numpy(case.hist).to(dev), clear_err=clear)
    out.err.fill_(err_fill)
    lib = _lib.load()
    _lib.check(lib.gr_beam_step(ctypes.byref(desc), ctypes.byref(io), ctypes.c_void_p(ws.data_ptr()),
                                ctypes.c_size_t(ws.numel()), ctypes.c_void_p(s.cuda_stream)), "gr_beam_step")
    torch.cuda.synchronize()
    return {k: getattr(out, k).cpu().numpy() for k in OUT_KEYS}, int(out.err.item())


def test_clear_flag_and_or_semantics():
    cat = small_catalog()
    R, NB, B, V = 3, 16, 16, 8192
    node = np.full((R, NB), cat.start_node, np.int32)
    case = Case(logits32=make_logits(R, NB, V, 4.0, 91, "bf16"), dtype="bf16", cum=initial_cum(R, NB),
                node=node, beam_width=B, vocab_size=V, csr=cat.csr,
                hist=np.full((R, NB, 1), cat.sid_begin, np.int32))
    ref, ref_err = _call(case, cat, node, 0, clear=False)
    assert ref_err == 0
    # a dirty word is cleared, and the outputs are the same bits
    got, err = _call(case, cat, node, 0x7F7F0000, clear=True)
    assert err == 0
    assert_bit_exact(got, ref)
    # without the flag the step ORs into the word as it stands
    _, err = _call(case, cat, node, 0x100, clear=False)
    assert err == 0x100
    # a node id out of range: reported once the word is cleared, the row treated as dead
    bad = node.copy()
    bad[1, 5] = cat.csr.num_nodes + 7
    dead = node.copy()
    dead[1, 5] = -2
    want, _ = _call(case, cat, dead, 0, clear=False)
    for clear, fill in ((True, 0x7F7F0000), (False, 0)):
        got, err = _call(case, cat, bad, fill, clear=clear)
        assert err == GR_DEVERR_BAD_NODE
        assert_bit_exact(got, want)
