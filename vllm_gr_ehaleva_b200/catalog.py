"""Item catalog as a CSR trie of semantic-ID token sequences.

Mirrors the reference's ``Catalog`` (vllm_gr/entrypoints/openai/serving_models.py:18-49):
``Catalog(tokenizer)``, ``load(path)`` reading a JSON list of token-string
lists, and ``valid(token_ids) -> set[int]`` walking the trie from its root.
Loading errors are the reference's ValueErrors.  Instead of a nested dict the
trie is kept as CSR arrays, which is what the device step reads:

    row_ptr    int64 [N+1]   children of node n are edges row_ptr[n]:row_ptr[n+1]
    child_tok  int32 [E]     edge token id, ascending within a node
    child_node int32 [E]     node reached over the edge

Node 0 is the root.  Nodes are numbered level by level (breadth first), and
within a level in lexicographic order of their prefix, so every node's edges
are contiguous and sorted by token.
"""
from __future__ import annotations

import json
from typing import Any, Iterable, Sequence

import numpy as np

NODE_UNCONSTRAINED = -1
NODE_DEAD = -2


class CSRTrie:
    """CSR trie arrays plus host-side walking helpers."""

    def __init__(self, row_ptr: np.ndarray, child_tok: np.ndarray, child_node: np.ndarray):
        self.row_ptr = np.ascontiguousarray(row_ptr, dtype=np.int64)
        self.child_tok = np.ascontiguousarray(child_tok, dtype=np.int32)
        self.child_node = np.ascontiguousarray(child_node, dtype=np.int32)
        if self.row_ptr.ndim != 1 or self.row_ptr.shape[0] < 1 or self.row_ptr[0] != 0:
            raise ValueError("row_ptr must start at 0")
        if self.row_ptr[-1] != self.child_tok.shape[0] or self.child_tok.shape != self.child_node.shape:
            raise ValueError("row_ptr / child arrays disagree on the edge count")

    @property
    def num_nodes(self) -> int:
        return int(self.row_ptr.shape[0] - 1)

    @property
    def num_edges(self) -> int:
        return int(self.child_tok.shape[0])

    def children(self, n: int) -> np.ndarray:
        return self.child_tok[self.row_ptr[n]:self.row_ptr[n + 1]]

    def degree(self, n) -> np.ndarray:
        n = np.asarray(n)
        return self.row_ptr[n + 1] - self.row_ptr[n]

    def step(self, n: int, tok: int) -> int:
        """Node reached from ``n`` over ``tok``; NODE_DEAD if there is no such edge."""
        if n == NODE_UNCONSTRAINED:
            return NODE_UNCONSTRAINED
        if n < 0:
            return NODE_DEAD
        a, b = int(self.row_ptr[n]), int(self.row_ptr[n + 1])
        i = a + int(np.searchsorted(self.child_tok[a:b], tok))
        if i < b and int(self.child_tok[i]) == tok:
            return int(self.child_node[i])
        return NODE_DEAD

    def walk(self, token_ids: Iterable[int], start: int = 0) -> int:
        n = start
        for t in token_ids:
            n = self.step(n, int(t))
            if n == NODE_DEAD:
                return NODE_DEAD
        return n

    def validate(self, vocab_size: int) -> None:
        """Host-side checks the device step relies on (sorted, in-range children)."""
        if self.num_edges:
            if self.child_tok.min() < 0 or self.child_tok.max() >= vocab_size:
                raise ValueError("catalog token id outside the vocabulary")
            if self.child_node.min() < 0 or self.child_node.max() >= self.num_nodes:
                raise ValueError("catalog child node id out of range")
            deg = np.diff(self.row_ptr)
            same = np.repeat(np.arange(self.num_nodes), deg)
            d = np.diff(self.child_tok.astype(np.int64))
            bad = (d <= 0) & (same[1:] == same[:-1])
            if bad.any():
                raise ValueError("catalog children must be strictly ascending per node")


def csr_from_sorted_unique(seqs: np.ndarray) -> CSRTrie:
    """Trie of equal-length token sequences given sorted (lexicographic) and unique."""
    seqs = np.asarray(seqs, dtype=np.int64)
    n, D = seqs.shape
    if n == 0:
        return CSRTrie(np.zeros(2, np.int64), np.zeros(0, np.int32), np.zeros(0, np.int32))
    new_prev = np.zeros(n, dtype=bool)
    new_prev[0] = True
    level_first = []            # per level d=1..D: boolean "row starts a new level-d prefix"
    for d in range(1, D + 1):
        col = seqs[:, d - 1]
        changed = np.empty(n, dtype=bool)
        changed[0] = True
        changed[1:] = col[1:] != col[:-1]
        new_d = new_prev | changed
        level_first.append(new_d)
        new_prev = new_d
    counts = [1] + [int(f.sum()) for f in level_first]
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int64)
    num_nodes = int(sum(counts))
    child_tok_parts, child_node_parts = [], []
    deg = np.zeros(num_nodes, dtype=np.int64)
    parent_rank_prev = np.zeros(n, dtype=np.int64)   # level-0 rank of every row: the root
    for d in range(1, D + 1):
        first = level_first[d - 1]
        rows = np.nonzero(first)[0]
        parents = offsets[d - 1] + parent_rank_prev[rows]
        child_tok_parts.append(seqs[rows, d - 1])
        child_node_parts.append(offsets[d] + np.arange(rows.shape[0], dtype=np.int64))
        _bincount_into(deg, parents)
        parent_rank_prev = np.cumsum(first) - 1
    row_ptr = np.concatenate([[0], np.cumsum(deg)]).astype(np.int64)
    child_tok = np.concatenate(child_tok_parts).astype(np.int32)
    child_node = np.concatenate(child_node_parts).astype(np.int32)
    return CSRTrie(row_ptr, child_tok, child_node)


def _bincount_into(deg: np.ndarray, parents: np.ndarray) -> None:
    lo, hi = int(parents.min()), int(parents.max())
    deg[lo:hi + 1] += np.bincount(parents - lo, minlength=hi - lo + 1)


def csr_from_sequences(seqs: Sequence[Sequence[int]]) -> CSRTrie:
    """Trie of token sequences of any lengths (duplicates allowed)."""
    seqs = [list(map(int, s)) for s in seqs]
    if seqs and all(len(s) == len(seqs[0]) for s in seqs):
        arr = np.asarray(seqs, dtype=np.int64).reshape(len(seqs), len(seqs[0]))
        if arr.shape[1] == 0:
            return CSRTrie(np.zeros(2, np.int64), np.zeros(0, np.int32), np.zeros(0, np.int32))
        arr = np.unique(arr, axis=0)
        return csr_from_sorted_unique(arr)
    # ragged: nested dict trie, then breadth-first numbering
    root: dict[int, Any] = {}
    for s in seqs:
        nd = root
        for t in s:
            nd = nd.setdefault(t, {})
    level = [root]
    row_ptr = [0]
    child_tok: list[int] = []
    child_node: list[int] = []
    next_id = 1
    while level:
        nxt = []
        for nd in level:
            for t in sorted(nd):
                child_tok.append(t)
                child_node.append(next_id)
                next_id += 1
                nxt.append(nd[t])
            row_ptr.append(len(child_tok))
        level = nxt
    return CSRTrie(np.asarray(row_ptr), np.asarray(child_tok), np.asarray(child_node))


class Catalog:
    """Drop-in for the reference ``Catalog`` backed by a CSR trie.

    ``load`` / ``valid`` keep the reference's behaviour and error messages
    (serving_models.py:23-49); ``csr`` is the device-ready form.
    """

    def __init__(self, tokenizer: Any):
        self.tokenizer = tokenizer
        self.csr: CSRTrie | None = None
        self._device_cache: dict = {}

    def load(self, path: str) -> None:
        try:
            with open(path) as f:
                catalog_data = json.load(f)
        except FileNotFoundError:
            raise ValueError(f"Catalog file not found: {path}")
        except json.JSONDecodeError:
            raise ValueError(f"Failed to decode JSON from catalog file: {path}")
        seqs = []
        for seq in catalog_data:
            token_ids = self.tokenizer.convert_tokens_to_ids(seq)
            for i, token_id in enumerate(token_ids):
                if token_id is None:
                    raise ValueError(f"Invalid token ID: {seq[i]} at index {i}")
            seqs.append([int(t) for t in token_ids])
        self.load_token_ids(seqs)

    def load_token_ids(self, seqs: Sequence[Sequence[int]]) -> None:
        self.csr = csr_from_sequences(seqs)
        self._device_cache.clear()

    def valid(self, token_ids: list[int]) -> set[int]:
        if self.csr is None:
            return set()
        n = self.csr.walk(token_ids)
        if n < 0:
            return set()
        return set(int(t) for t in self.csr.children(n))

    def node_of(self, token_ids: Iterable[int]) -> int:
        """Trie node after ``token_ids`` (NODE_DEAD if the prefix is not in the catalog)."""
        if self.csr is None:
            return NODE_UNCONSTRAINED
        return self.csr.walk(token_ids)

    def device_arrays(self, device):
        """(row_ptr, child_tok, child_node) as torch tensors on ``device`` (cached)."""
        import torch
        key = str(device)
        if key not in self._device_cache:
            c = self.csr
            self._device_cache[key] = (
                torch.from_numpy(c.row_ptr).to(device),
                torch.from_numpy(c.child_tok).to(device),
                torch.from_numpy(c.child_node).to(device),
            )
        return self._device_cache[key]
