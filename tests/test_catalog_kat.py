"""Catalog trie: the reference's known-answer test (tests/test_catalog.py:29-65)
ported to the CSR catalog, plus CSR invariants the device step relies on."""
import json
import os
import tempfile
from unittest.mock import MagicMock

import numpy as np
import pytest

from vllm_gr_ehaleva_b200.catalog import Catalog, csr_from_sequences
from vllm_gr_ehaleva_b200.synthetic import make_catalog


@pytest.fixture
def mock_tokenizer():
    tok = MagicMock()

    def convert_tokens_to_ids(seq):
        if isinstance(seq, list):
            return [int(x) for x in seq]
        return int(seq)

    tok.convert_tokens_to_ids.side_effect = convert_tokens_to_ids
    return tok


def test_catalog_functionality(mock_tokenizer):
    data = [["1", "2", "3", "4", "5"], ["1", "2", "3", "6", "7"], ["8", "9", "10", "11", "12"]]
    with tempfile.NamedTemporaryFile(mode="w", delete=False, suffix=".json") as f:
        json.dump(data, f)
        path = f.name
    try:
        cat = Catalog(mock_tokenizer)
        cat.load(path)
        assert cat.valid([]) == {1, 8}
        assert cat.valid([1, 2, 3]) == {4, 6}
        assert cat.valid([1, 2, 3, 4]) == {5}
        assert cat.valid([1, 2, 3, 4, 5]) == set()
        assert cat.valid([99]) == set()
        assert cat.valid([1, 99]) == set()
    finally:
        os.remove(path)


def test_catalog_load_errors(mock_tokenizer):
    cat = Catalog(mock_tokenizer)
    with pytest.raises(ValueError, match="Catalog file not found"):
        cat.load("/nonexistent/catalog.json")
    with tempfile.NamedTemporaryFile(mode="w", delete=False, suffix=".json") as f:
        f.write("{not json")
        path = f.name
    try:
        with pytest.raises(ValueError, match="Failed to decode JSON"):
            cat.load(path)
    finally:
        os.remove(path)


def test_ragged_and_duplicate_sequences():
    seqs = [[1, 2], [1, 2, 3], [4], [1, 2]]
    csr = csr_from_sequences(seqs)
    assert set(csr.children(0).tolist()) == {1, 4}
    assert csr.children(csr.walk([1, 2])).tolist() == [3]
    assert csr.walk([4, 5]) == -2


def test_csr_invariants_on_synthetic_catalog():
    cat = make_catalog(20000, 3, 64, 4096, 1.1, seed=1)
    csr = cat.csr
    csr.validate(4096)
    # children strictly ascending, breadth-first node ids, every item reachable
    assert np.all(np.diff(csr.row_ptr) >= 0)
    assert csr.child_node.min() == 1 and csr.child_node.max() == csr.num_nodes - 1
    rng = np.random.default_rng(0)
    nodes = rng.integers(0, csr.num_nodes, 200)
    for n in nodes:
        kids = csr.children(n)
        assert np.all(np.diff(kids) > 0)
    # leaves = items (one <|sid_end|> edge each)
    leaves = np.nonzero(np.diff(csr.row_ptr) == 0)[0]
    assert leaves.shape[0] == cat.num_items
    # token layout: level l codes occupy [V - L*C + l*C, ...)
    kids = csr.children(cat.start_node)
    assert kids.min() >= 4096 - 3 * 64 and kids.max() < 4096 - 2 * 64
