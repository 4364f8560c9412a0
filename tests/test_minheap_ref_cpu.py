"""The candidate selection against the reference's own native code.

The reference ships a C++ bounded top-N over B per-beam candidate lists
(vllm_gr/csrc/minheap.cpp:75-114, MinHeapTuple.push_candidates_striped: EOS
entries skipped, a beam's list dropped as soon as one of its entries fails to
enter the heap).  oracle/Makefile compiles it from its source into
oracle/_ref/ (build() does so where the reference checkout is present); these
tests load it and require the same top-N set as the oracle's canonical top-k
(oracle/restated.py topk_canonical) on the same candidates, scores distinct.
Skipped where the module was not built."""
import glob
import importlib.util
import os

import numpy as np
import pytest

from oracle import restated as O

HERE = os.path.dirname(os.path.abspath(__file__))
_SO = glob.glob(os.path.join(os.path.dirname(HERE), "oracle", "_ref", "minheap_cpp*.so"))


def _module():
    if not _SO:
        pytest.skip("oracle/_ref/minheap_cpp not built (needs the reference checkout)")
    spec = importlib.util.spec_from_file_location("minheap_cpp", _SO[0])
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


@pytest.mark.parametrize("seed", range(8))
def test_striped_top_n_equals_canonical_top_k(seed):
    mh = _module()
    rng = np.random.default_rng(seed)
    B = int(rng.choice([4, 16, 128]))
    K = int(rng.choice([B, B + 1]))
    eos = 7
    cum = np.sort(rng.uniform(-20, 0, B).astype(np.float32))[::-1]
    # each beam's candidates sorted descending (log-probs of its top-K), some of them EOS
    lp = -np.sort(rng.exponential(3.0, (B, K)).astype(np.float32), axis=1)
    scores = (cum[:, None] + lp).astype(np.float32)
    toks = rng.integers(8, 150000, (B, K)).astype(np.int64)
    toks[rng.random((B, K)) < 0.05] = eos
    flat_scores, flat_toks = scores.ravel(), toks.ravel()
    N = 2 * B
    h = mh.MinHeapTuple(N)
    h.push_candidates_striped(flat_scores, flat_toks, K, eos)
    ref = sorted(idx for _, idx in h.items())
    keep = np.nonzero(flat_toks != eos)[0]
    ours = sorted(keep[O.topk_canonical(flat_scores[keep], keep.astype(np.int64), N)].tolist())
    assert ref == ours
