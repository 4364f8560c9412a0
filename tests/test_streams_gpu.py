"""The step on a caller-given side stream.

beam_step(..., stream=s) launches the library on `s` while the caller made
its inputs (and the front end its converted copies and outputs) on the
current stream.  The launch stream must wait for that work, and every tensor
the kernels read or write must stay allocated until they are done, even when
the caller drops its references right after the call.  Here the inputs become
ready only behind a long queue of matrix products on the current stream, the
cumulative scores need a dtype conversion inside the call, and the caller
frees its tensors and fills new ones of the same size at once: the outputs
must equal a plain call's bit for bit.
"""
import numpy as np
import pytest

from helpers import OUT_KEYS, Case, assert_bit_exact, gpu_step, make_logits, small_catalog, to_device_logits
from vllm_gr_ehaleva_b200.synthetic import initial_cum

pytestmark = pytest.mark.gpu


def test_side_stream_under_concurrent_load():
    import torch
    from vllm_gr_ehaleva_b200.sample import beam_step
    cat = small_catalog()
    R, NB, B, V = 3, 16, 16, 8192
    case = Case(logits32=make_logits(R, NB, V, 4.0, 61, "bf16"), dtype="bf16", cum=initial_cum(R, NB),
                node=np.full((R, NB), cat.start_node, np.int32), beam_width=B, vocab_size=V, csr=cat.csr,
                hist=np.full((R, NB, 1), cat.sid_begin, np.int32))
    ref = gpu_step(case)                                   # a plain call on the current stream
    dev = torch.device("cuda")
    src = to_device_logits(case, dev)
    csr = tuple(torch.from_numpy(a).to(dev) for a in (cat.csr.row_ptr, cat.csr.child_tok, cat.csr.child_node))
    side = torch.cuda.Stream(device=dev)
    for trial in range(3):
        a = torch.randn(4096, 4096, device=dev)
        for _ in range(16):                                # a long queue ahead of the inputs
            a = a @ a
            a = a / a.norm()
        logits = torch.empty_like(src)
        logits.copy_(src)
        cum64 = torch.from_numpy(case.cum).to(dev, torch.float64)   # converted inside the call
        node = torch.from_numpy(case.node).to(dev)
        hist = torch.from_numpy(case.hist).to(dev)
        out = beam_step(logits, cum64, node, beam_width=B, csr=csr, vocab_size=V, hist=hist, stream=side)
        # the caller lets go of its inputs at once and reuses the memory
        del logits, cum64, node, hist, a
        junk = [torch.full_like(src, 3.0) for _ in range(2)] + [torch.full((R, NB), 9.0, device=dev)]
        side.synchronize()
        got = {k: getattr(out, k).cpu().numpy() for k in OUT_KEYS}
        got["err"] = int(out.err.item())
        assert got["err"] == 0
        assert_bit_exact(got, ref)
        del junk
