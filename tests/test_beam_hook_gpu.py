"""The worker hook on the GPU: sessions stepped in runs over the worker's row
layout (plain rows and chunked prefills in between) give exactly what a
separate step call per session gives, and the device-resident state carries
over to the next step."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from helpers import small_catalog  # noqa: E402
from vllm_gr_ehaleva_b200.engine import WorkerBeamHook  # noqa: E402
from vllm_gr_ehaleva_b200.sample import beam_step  # noqa: E402
from vllm_gr_ehaleva_b200.synthetic import initial_cum  # noqa: E402

DEV = "cuda"


def test_hook_matches_per_session_steps_over_two_steps():
    V = 8192
    cat = small_catalog(V=V)
    csr = tuple(torch.from_numpy(a).to(DEV) for a in (cat.csr.row_ptr, cat.csr.child_tok, cat.csr.child_node))
    widths = {"a": 16, "b": 16, "c": 8, "d": 16}
    hook = WorkerBeamHook(vocab_size=V, csr=csr, eos_token_id=None, device=DEV)
    ref_state = {}
    for i, (r, B) in enumerate(widths.items()):
        cum = torch.from_numpy(initial_cum(1, B)[0]).to(DEV)
        node = torch.full((B,), cat.start_node, dtype=torch.int32, device=DEV)
        hook.start(r, B, cum, node)
        ref_state[r] = (cum.clone(), node.clone(), None)
    cfg = [("a", 0, 16), ("b", 1, 16), ("plain", 2, 1), ("prefill", 3, 0), ("c", 4, 8), ("d", 5, 16)]
    rows = sum(w for _, _, w in cfg)
    g = torch.Generator(device=DEV).manual_seed(3)
    for step in range(2):
        logits = (torch.randn(rows, V, device=DEV, generator=g) * 4).to(torch.bfloat16)
        got = hook.step(logits, cfg)
        assert set(got) == set(widths)
        row = 0
        for r, _, w in cfg:
            if r in widths:
                cum, node, hist = ref_state[r]
                out = beam_step(logits[row:row + w], cum[None], node[None], beam_width=w, csr=csr, vocab_size=V,
                                hist=None if hist is None else hist[None])
                for k in ("sel_parent", "sel_token", "sel_node"):
                    assert torch.equal(getattr(got[r], k), getattr(out, k)[0]), (step, r, k)
                assert torch.equal(got[r].sel_score.view(torch.int32), out.sel_score[0].view(torch.int32))
                assert torch.equal(got[r].hist, out.hist_out[0])
                ref_state[r] = (out.sel_score[0].clone(), out.sel_node[0].clone(), out.hist_out[0].clone())
            row += w
    assert hook.sessions["a"].hist.shape == (16, 2)
    hook.end("a")
    assert "a" not in hook.sessions
