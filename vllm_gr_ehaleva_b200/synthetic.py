"""Seeded synthetic inputs with the shapes of the reference's workloads.

The reference's own benchmark data (OpenOneRec dataset, OneRec model) is not
available; these generators stand in for it with the shapes its tools use:
semantic IDs of L codes drawn from codebooks of C codes each, mapped to
disjoint token-id ranges at the tail of the vocabulary, wrapped in
``<|sid_begin|> ... <|sid_end|>`` tokens like the reference's catalog
converter (benchmarks/open_one_rec/tools/convert_catalog.py:14-29).

Token layout for vocabulary V, L levels, codebook C:
    level l code c          -> V - L*C + l*C + c          (l = 0..L-1)
    <|sid_begin|>           -> V - L*C - 2
    <|sid_end|>             -> V - L*C - 1
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .catalog import CSRTrie, csr_from_sorted_unique


@dataclass
class SyntheticCatalog:
    csr: CSRTrie
    vocab_size: int
    levels: int
    codebook: int
    num_items: int          # distinct items after de-duplication
    sid_begin: int
    sid_end: int
    start_node: int         # trie node after <|sid_begin|>: where every beam starts

    def level_token(self, level: int, code):
        return self.vocab_size - self.levels * self.codebook + level * self.codebook + np.asarray(code)


def make_catalog(num_items: int, levels: int, codebook: int, vocab_size: int,
                 zipf_a: float, seed: int = 1) -> SyntheticCatalog:
    """Catalog of ``num_items`` draws: level-1 code ~ Zipf(zipf_a) truncated to the
    codebook, deeper codes uniform; duplicate items removed."""
    rng = np.random.default_rng(seed)
    C, L, V = int(codebook), int(levels), int(vocab_size)
    if L * C + 2 > V:
        raise ValueError("semantic-ID tail does not fit in the vocabulary")
    k = np.arange(1, C + 1, dtype=np.float64)
    p = k ** (-float(zipf_a))
    p /= p.sum()
    codes = np.empty((num_items, L), dtype=np.int64)
    codes[:, 0] = rng.choice(C, size=num_items, p=p)
    if L > 1:
        codes[:, 1:] = rng.integers(0, C, size=(num_items, L - 1))
    bits = int(np.ceil(np.log2(C)))
    if bits * L > 62:
        raise ValueError("catalog too deep to encode")
    key = np.zeros(num_items, dtype=np.int64)
    for lvl in range(L):
        key = (key << bits) | codes[:, lvl]
    key = np.unique(key)
    n = key.shape[0]
    uniq = np.empty((n, L), dtype=np.int64)
    for lvl in range(L - 1, -1, -1):
        uniq[:, lvl] = key & ((1 << bits) - 1)
        key = key >> bits
    base = V - L * C
    sid_begin, sid_end = base - 2, base - 1
    seqs = np.empty((n, L + 2), dtype=np.int64)
    seqs[:, 0] = sid_begin
    seqs[:, 1:L + 1] = base + np.arange(L, dtype=np.int64)[None, :] * C + uniq
    seqs[:, L + 1] = sid_end
    csr = csr_from_sorted_unique(seqs)            # rows already sorted: same prefix, sorted codes
    start = csr.step(0, sid_begin)
    return SyntheticCatalog(csr=csr, vocab_size=V, levels=L, codebook=C, num_items=n,
                            sid_begin=sid_begin, sid_end=sid_end, start_node=start)


def initial_cum(num_requests: int, num_beams: int, seed: int = 2) -> np.ndarray:
    """Initial cumulative beam scores ~ U[-20, 0], sorted descending per request."""
    rng = np.random.default_rng(seed)
    c = rng.uniform(-20.0, 0.0, size=(num_requests, num_beams)).astype(np.float32)
    return -np.sort(-c, axis=1)


def histories(num_requests: int, num_beams: int, length: int, vocab_size: int,
              seed: int = 3) -> np.ndarray:
    """Per-beam prior-token histories drawn uniformly from the vocabulary."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, vocab_size, size=(num_requests, num_beams, length)).astype(np.int32)


def logits_numpy(rows: int, cols: int, sigma: float, seed: int) -> np.ndarray:
    """float32 logits ~ N(0, sigma^2) on the host (for CPU-side cases)."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(sigma)).astype(np.float32)


def logits_torch(rows: int, cols: int, sigma: float, seed: int, dtype, device):
    """Logits ~ N(0, sigma^2) generated on ``device`` with a seeded torch.Generator,
    then cast to ``dtype`` (bf16 rounding happens after the fp32 draw)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    x = torch.randn((rows, cols), generator=g, device=device, dtype=torch.float32)
    x.mul_(float(sigma))
    return x.to(dtype)


# BASELINE.json configs (index 1-based as in the prose: cfg1 .. cfg5)
CONFIGS = {
    "cfg1": dict(requests=1, beams=128, vocab=152064, dtype="f32", sigma=4.0, items=100_000,
                 levels=3, codebook=8192, zipf=1.1, steps=3, mode="raw"),
    "cfg2": dict(requests=32, beams=128, vocab=152064, dtype="bf16", sigma=4.0, items=1_000_000,
                 levels=3, codebook=8192, zipf=1.1, steps=3, mode="raw"),
    "cfg3": dict(requests=128, beams=512, vocab=152064, dtype="bf16", sigma=4.0, items=10_000_000,
                 levels=4, codebook=4096, zipf=1.2, steps=4, mode="raw"),
    "cfg4": dict(requests=64, beams=256, vocab=152064, dtype="f32", sigma=3.0, items=0,
                 levels=0, codebook=0, zipf=0.0, steps=8, mode="processed", temperature=0.7,
                 rep=1.2, pres=0.5, freq=0.0, hist=64),
    "cfg5": dict(requests=8, beams=1024, vocab=152064, dtype="bf16", sigma=4.0, items=1_000_000,
                 levels=3, codebook=8192, zipf=1.1, steps=3, mode="raw", shards=8),
}
