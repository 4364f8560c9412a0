"""CPU restatement of the reference's logprobs remux (TEST INFRASTRUCTURE).

Follows vllm_gr/v1/engine/engine_core_patch.py:383-445
(_remux_logprobs_tensors): the sampler's per-row outputs of each mega request
(W rows of K logprobs / token ids and W ranks) become one row of W*K entries,
padded to the widest request (-inf for logprobs, 0 for ids and ranks); a
request with no row (an intermediate chunked prefill) gets an all-padding row
and sampled id -1; the sampled-token column keeps the request's first row.
Pinned by tests/golden/remux_cases.json (the reference run itself).
"""
from __future__ import annotations

import numpy as np


def remux(ws, max_dim, K, lps, ids, ranks, st):
    n = len(ws)
    out_lps = np.full((n, max_dim), -np.inf, np.float32)
    out_ids = None if ids is None else np.zeros((n, max_dim), ids.dtype)
    out_ranks = None if ranks is None else np.zeros((n, max_dim), ranks.dtype)
    out_st = np.full((n, st.shape[1]), -1, st.dtype)
    cur = 0
    for c, w in enumerate(ws):
        if w == 0:
            continue
        out_st[c] = st[cur]
        out_lps[c, :w * K] = lps[cur:cur + w, :K].reshape(-1)
        if ids is not None:
            out_ids[c, :w * K] = ids[cur:cur + w, :K].reshape(-1)
        if ranks is not None:
            out_ranks[c, :w] = ranks[cur:cur + w]
        cur += w
    return out_st, out_lps, out_ids, out_ranks


def remux_torch(ws, max_dim, K, lps, ids, ranks, st):
    """The same remux as per-request torch slices, pads and one cat (the
    reference's way, on whatever device the tensors are): the timing baseline."""
    import torch
    sts, ls, is_, rs = [], [], [], []
    cur = 0
    for w in ws:
        if w == 0:
            sts.append(torch.full((1, 1), -1, dtype=st.dtype, device=st.device))
            ls.append(torch.full((1, max_dim), float("-inf"), dtype=lps.dtype, device=lps.device))
            is_.append(torch.zeros((1, max_dim), dtype=ids.dtype, device=ids.device))
            rs.append(torch.zeros((1, max_dim), dtype=ranks.dtype, device=ranks.device))
            continue
        sts.append(st[cur:cur + 1])
        pad = max_dim - w * K
        ls.append(torch.nn.functional.pad(lps[cur:cur + w, :K].reshape(1, -1), (0, pad), value=float("-inf")))
        is_.append(torch.nn.functional.pad(ids[cur:cur + w, :K].reshape(1, -1), (0, pad), value=0))
        rs.append(torch.nn.functional.pad(ranks[cur:cur + w].reshape(1, -1), (0, max_dim - w), value=0))
        cur += w
    return torch.cat(sts), torch.cat(ls), torch.cat(is_), torch.cat(rs)
