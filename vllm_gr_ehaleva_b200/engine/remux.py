"""Per-request remux of the sampler's logprob rows (CUDA, one launch).

Drop-in for the reference's _remux_logprobs_tensors
(vllm_gr/v1/engine/engine_core_patch.py:383-445): same arguments, same four
results.  The mega request that owns W logit rows gets one row of W*K
logprobs / token ids (its rows in order) and W ranks, padded to
max_chained_dim with -inf / 0 / 0; a request with no row (an intermediate
chunked prefill) gets an all-padding row and sampled id -1; the sampled-token
column keeps each request's first row.  The reference builds this with a
Python loop of slices, pads and a cat per call; here the per-request offsets
are computed on the host (O(requests)) and gr_remux_logprobs writes every row.
"""
from __future__ import annotations

import ctypes

from .. import _lib


def remux_logprobs_tensors(request_row_configs, max_chained_dim, target_K, orig_lps, orig_lp_ids, orig_ranks,
                           st_ids):
    """request_row_configs: [(req_id, input_row, W_logits)]; orig_lps: float32
    [rows, >= target_K] (CUDA); orig_lp_ids: int [rows, >= target_K] or None;
    orig_ranks: int [rows] or None; st_ids: int [rows, 1].  Returns
    (st_ids, logprobs, logprob_token_ids, ranks) as the reference does."""
    import torch
    if max_chained_dim == 0 or orig_lps.numel() == 0:
        return st_ids, orig_lps, orig_lp_ids, orig_ranks
    ws = [int(w) for _, _, w in request_row_configs]
    K, max_dim, rows = int(target_K), int(max_chained_dim), int(orig_lps.shape[0])
    if orig_lps.dtype != torch.float32 or orig_lps.dim() != 2 or orig_lps.stride(1) != 1:
        raise ValueError("orig_lps must be a float32 [rows, K] tensor with unit column stride")
    if K <= 0 or K > orig_lps.shape[1]:
        raise ValueError(f"target_K={K} outside [1, {orig_lps.shape[1]}]")
    if any(w < 0 for w in ws) or sum(ws) > rows or max(ws) * K > max_dim:
        raise ValueError("W_logits do not fit the sampler rows or max_chained_dim")
    if st_ids.dim() != 2 or st_ids.shape[1] != 1:
        raise ValueError("st_ids must be [rows, 1]")
    dev = orig_lps.device
    starts, cur = [], 0
    for w in ws:
        starts.append(cur)
        cur += w
    n = len(ws)
    row_w = torch.tensor(ws, dtype=torch.int32).to(dev)
    row_start = torch.tensor(starts, dtype=torch.int64).to(dev)
    out_lps = torch.empty((n, max_dim), dtype=torch.float32, device=dev)
    out_st = torch.empty((n, 1), dtype=st_ids.dtype, device=dev)
    ids = None if orig_lp_ids is None else orig_lp_ids
    if ids is not None and (ids.dim() != 2 or ids.stride(1) != 1 or ids.shape[1] < K):
        raise ValueError("orig_lp_ids must be [rows, >= K] with unit column stride")
    ranks = None if orig_ranks is None else orig_ranks.contiguous()
    out_ids = None if ids is None else torch.empty((n, max_dim), dtype=ids.dtype, device=dev)
    out_ranks = None if ranks is None else torch.empty((n, max_dim), dtype=ranks.dtype, device=dev)
    d = _lib.RemuxDesc()
    d.num_requests, d.K, d.max_dim, d.num_rows = n, K, max_dim, rows
    d.lps_stride = orig_lps.stride(0)
    d.ids_stride = 0 if ids is None else ids.stride(0)
    d.st_stride = st_ids.stride(0)
    d.ids_bytes = 0 if ids is None else ids.element_size()
    d.ranks_bytes = 0 if ranks is None else ranks.element_size()
    d.st_bytes = st_ids.element_size()

    def ptr(t):
        return None if t is None else t.data_ptr()

    lib = _lib.load()
    rc = lib.gr_remux_logprobs(d, row_w.data_ptr(), row_start.data_ptr(), orig_lps.data_ptr(), ptr(ids), ptr(ranks),
                               st_ids.data_ptr(), out_lps.data_ptr(), ptr(out_ids), ptr(out_ranks),
                               out_st.data_ptr(), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    if rc != _lib.GR_OK:
        raise RuntimeError(f"gr_remux_logprobs failed: {_lib.STATUS_NAMES.get(rc, rc)}")
    return out_st, out_lps, out_ids, out_ranks
