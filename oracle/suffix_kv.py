"""CPU restatement of the reference's suffix KV pass (TEST INFRASTRUCTURE).

Only tests/ import this; the product path is the CUDA gather behind
gr_suffix_kv_gather (vllm_gr_ehaleva_b200/attention/suffix_kv.py).

Follows vllm_gr/v1/attention/backends/beam_attn.py:
  * suffix_metadata: BeamAttentionMetadataBuilder._segment_requests (255-292)
    and the suffix part of _build_mega_mappings (319-413): which query tokens
    of a mega-decode request go to the prefix pass, and for every beam the list
    of positions (into those tokens) that make up its suffix: beam 0 its own
    tokens, beams 1.. the request's uncached prefix tail followed by their own;
  * gather: paged_kv_to_contig_suffix_kernel / extract_suffix_kv (62-117):
    out[t] = cache[slot_mapping[slot_mapping_out[t]]] for K and V, a flat slot
    addressing token slot * stride(1) of the cache.
Pinned against the reference builder's own outputs
(tests/golden/suffix_metadata.json, written by tests/golden/make_suffix_golden.py).
"""
from __future__ import annotations

import numpy as np


def suffix_metadata(mega, q_starts, block_size):
    """mega: per request index i, None (a standard request) or a dict with
    prefix_len, cache_len, beam_width, steps.  q_starts: query start offsets
    (len num_reqs + 1).  Returns (mega_prefix_indices, slot_mapping_out,
    suffix_q_lens, suffix_seq_lens)."""
    num_reqs = len(q_starts) - 1
    rows = []   # (req, prefix_len, beam_width, steps, cache_len, q_offset)
    for i in range(num_reqs):
        m = mega[i] if i < len(mega) else None
        if not m:
            continue
        prefix_len, cache_len = m["prefix_len"], m["cache_len"]
        delta = prefix_len - cache_len
        q_offset = 0
        if delta > 0 and delta >= 2 * block_size:
            # a long uncached prefix runs through standard attention first (255-292)
            std_q_len = min(delta, q_starts[i + 1] - q_starts[i])
            cache_len += std_q_len
            q_offset = std_q_len
        rows.append((i, prefix_len, m["beam_width"], m["steps"], cache_len, q_offset))

    prefix_indices, smo, q_lens, seq_lens = [], [], [], []
    out_slot = 0
    for req, prefix_len, w, steps, cache_len, q_offset in rows:
        q_start = q_starts[req] + q_offset
        q_len = q_starts[req + 1] - q_start
        if w == 0 or steps == 0 or q_len <= 0:
            continue
        remaining = prefix_len - cache_len
        assert remaining >= 0
        shared = np.arange(out_slot, out_slot + remaining)
        budget = q_len
        q_cur = q_start
        group_len = 0
        for b in range(w):
            if budget <= 0:
                break
            if b == 0:
                own = min(budget, remaining + steps)
                seq = own
            else:
                own = min(budget, steps)
                seq = remaining + own
            if own <= 0:
                continue
            if b == 0:
                smo.extend(range(out_slot, out_slot + own))
            else:
                smo.extend(shared.tolist())
                smo.extend(range(out_slot, out_slot + own))
            q_lens.append(own)
            seq_lens.append(seq)
            group_len += own
            budget -= own
            out_slot += own
        if group_len:
            prefix_indices.extend(range(q_cur, q_cur + group_len))
    return (np.asarray(prefix_indices, np.int64), np.asarray(smo, np.int32), np.asarray(q_lens, np.int32),
            np.asarray(seq_lens, np.int32))


def gather(k_cache: np.ndarray, v_cache: np.ndarray, slot_mapping: np.ndarray, slot_mapping_out: np.ndarray,
           n: int):
    """k_cache / v_cache: [num_blocks, block_size, heads, dim] (contiguous).
    Returns out_k, out_v: [n, heads, dim]."""
    H, D = k_cache.shape[2], k_cache.shape[3]
    slots = slot_mapping[slot_mapping_out[:n].astype(np.int64)]
    return k_cache.reshape(-1, H, D)[slots], v_cache.reshape(-1, H, D)[slots]
