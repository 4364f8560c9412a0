"""Suffix KV gather of the beam-consecutive attention pass (CUDA, sm_100a).

Drop-in for the reference's Triton launcher
vllm_gr/v1/attention/backends/beam_attn.py:97-117 (extract_suffix_kv): same
arguments, same result, through gr_suffix_kv_gather of the C ABI.  For every
output token t, out_k[t] = k_cache[slot_mapping[slot_mapping_out[t]]] (all KV
heads and the head dimension), the flat slot addressing token `slot *
k_cache.stride(1)` as the reference kernel does; the same for V.  The reference
reads whatever memory an out-of-range index points at; here such tokens give
zero rows and set GR_DEVERR_BAD_SLOT in `err` when an error word is passed.
"""
from __future__ import annotations

from .. import _lib


def _slot_capacity(cache, heads: int, dim: int) -> int:
    """Flat slots that the reference's addressing can reach inside the cache's
    storage: at most num_blocks * block_size, and no slot whose row ends past
    the end of the storage."""
    n = cache.shape[0] * cache.shape[1]
    st, sh, sd = cache.stride(1), cache.stride(2), cache.stride(3)
    extent = cache.untyped_storage().nbytes() // cache.element_size() - cache.storage_offset()
    inner = (heads - 1) * sh + (dim - 1) * sd + 1
    if st > 0:
        n = min(n, (extent - inner) // st + 1)
    return max(int(n), 0)


def gather_desc(k_cache, v_cache, slot_mapping, slot_mapping_out, out_token_num: int) -> _lib.KvGatherDesc:
    """The call's descriptor (host only; raises ValueError on inconsistent arguments)."""
    if k_cache.dim() != 4 or v_cache.dim() != 4:
        raise ValueError("k_cache / v_cache must be [num_blocks, block_size, num_kv_heads, head_dim]")
    if k_cache.dtype != v_cache.dtype or k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache must have the same dtype and shape")
    if k_cache.element_size() not in (1, 2, 4):
        raise ValueError(f"unsupported KV element size {k_cache.element_size()}")
    if any(s < 0 for s in tuple(k_cache.stride()) + tuple(v_cache.stride())):
        raise ValueError("negative strides are not supported")
    n = int(out_token_num)
    if n < 0 or n > slot_mapping_out.numel():
        raise ValueError(f"out_token_num={n} exceeds slot_mapping_out ({slot_mapping_out.numel()} entries)")
    heads, dim = int(k_cache.shape[2]), int(k_cache.shape[3])
    d = _lib.KvGatherDesc()
    d.num_out = n
    d.num_src = int(slot_mapping.numel())
    d.num_slots = min(_slot_capacity(k_cache, heads, dim), _slot_capacity(v_cache, heads, dim))
    d.num_heads, d.head_dim, d.elem_bytes = heads, dim, int(k_cache.element_size())
    d.k_stride_tok, d.k_stride_head, d.k_stride_dim = k_cache.stride(1), k_cache.stride(2), k_cache.stride(3)
    d.v_stride_tok, d.v_stride_head, d.v_stride_dim = v_cache.stride(1), v_cache.stride(2), v_cache.stride(3)
    return d


def extract_suffix_kv(k_cache, v_cache, slot_mapping, slot_mapping_out, out_token_num, *, err=None):
    """Returns (out_k, out_v), each [out_token_num, num_kv_heads, head_dim] in the
    cache's dtype.  slot_mapping: flat cache slots (int64, int32 is widened);
    slot_mapping_out: int32 positions into slot_mapping; err: optional int32
    device tensor that receives GR_DEVERR_* bits.  Runs on the current stream."""
    import torch
    d = gather_desc(k_cache, v_cache, slot_mapping, slot_mapping_out, out_token_num)
    heads, dim = d.num_heads, d.head_dim
    out_k = torch.empty((d.num_out, heads, dim), device=k_cache.device, dtype=k_cache.dtype)
    out_v = torch.empty((d.num_out, heads, dim), device=v_cache.device, dtype=v_cache.dtype)
    if d.num_out == 0:
        return out_k, out_v
    lib = _lib.load()
    sm = slot_mapping if slot_mapping.dtype == torch.int64 else slot_mapping.to(torch.int64)
    smo = slot_mapping_out if slot_mapping_out.dtype == torch.int32 else slot_mapping_out.to(torch.int32)
    sm, smo = sm.contiguous(), smo.contiguous()
    if err is not None and (err.dtype != torch.int32 or not err.is_cuda):
        raise ValueError("err must be an int32 CUDA tensor")
    stream = torch.cuda.current_stream(k_cache.device).cuda_stream
    rc = lib.gr_suffix_kv_gather(d, k_cache.data_ptr(), v_cache.data_ptr(), sm.data_ptr(), smo.data_ptr(),
                                 out_k.data_ptr(), out_v.data_ptr(), None if err is None else err.data_ptr(),
                                 stream)
    if rc != _lib.GR_OK:
        raise RuntimeError(f"gr_suffix_kv_gather failed: {_lib.STATUS_NAMES.get(rc, rc)}")
    return out_k, out_v


# ---------------------------------------------------------------- suffix metadata
def suffix_records(mega, q_starts, block_size: int):
    """Per-request records of the suffix pass (host, O(1) per request).

    `mega[i]` is None for a standard request or a dict with prefix_len,
    cache_len, beam_width and steps (the reference's mega_data entry);
    `q_starts` are the batch's query start offsets (len num_reqs + 1).  Follows
    the per-request arithmetic of the reference builder
    (vllm_gr/v1/attention/backends/beam_attn.py:255-292 and 319-413): a long
    uncached prefix (>= 2 blocks) first goes through standard attention; beam 0
    then takes min(q_len, remaining + steps) query tokens and every later beam
    `steps` until the request's query budget runs out.
    Returns (records, totals) with totals = dict(beams, prefix, suffix, max_q, max_k)."""
    recs = []
    out_base = suffix_base = beam_base = 0
    max_q = max_k = 0
    for i in range(len(q_starts) - 1):
        m = mega[i] if i < len(mega) else None
        if not m:
            continue
        prefix_len, cache_len = int(m["prefix_len"]), int(m["cache_len"])
        w, steps = int(m["beam_width"]), int(m["steps"])
        q_offset = 0
        delta = prefix_len - cache_len
        if delta > 0 and delta >= 2 * block_size:
            std_q_len = min(delta, q_starts[i + 1] - q_starts[i])
            cache_len += std_q_len
            q_offset = std_q_len
        q_start = q_starts[i] + q_offset
        q_len = q_starts[i + 1] - q_start
        if w == 0 or steps == 0 or q_len <= 0:
            continue
        remaining = prefix_len - cache_len
        if remaining < 0:
            raise ValueError(f"request {i}: prefix_len {prefix_len} < cache_len {cache_len}")
        own0 = min(q_len, remaining + steps)
        extra = min(q_len - own0, (w - 1) * steps)
        beams = 1 + (extra + steps - 1) // steps
        seq_total = own0 + (beams - 1) * remaining + extra
        recs.append((q_start, out_base, suffix_base, beam_base, beams, remaining, steps, own0, own0 + extra))
        max_q = max(max_q, own0, min(steps, extra))
        max_k = max(max_k, own0, remaining + min(steps, extra) if extra else 0)
        out_base += own0 + extra
        suffix_base += seq_total
        beam_base += beams
    return recs, dict(beams=beam_base, prefix=out_base, suffix=suffix_base, max_q=max_q, max_k=max_k)


def build_suffix_metadata(mega, q_starts, block_size: int, device, *, err=None):
    """The suffix-pass metadata of the reference's BeamAttentionMetadataBuilder
    (mega_prefix_indices, mega_suffix_slot_mapping_out, mega_suffix_cu_seqlens_q
    / _k, mega_suffix_seq_lens and the maxima / total), with the per-beam and
    per-token arrays written on the device by gr_suffix_metadata instead of
    Python loops.  Returns a dict of device tensors and ints."""
    import ctypes

    import torch
    recs, tot = suffix_records(mega, q_starts, block_size)
    i64 = dict(dtype=torch.int64, device=device)
    i32 = dict(dtype=torch.int32, device=device)
    out = {"mega_prefix_indices": torch.empty(tot["prefix"], **i64),
           "suffix_slot_mapping_out": torch.empty(tot["suffix"], **i32),
           "suffix_cu_seqlens_q": torch.empty(tot["beams"] + 1, **i32),
           "suffix_cu_seqlens_k": torch.empty(tot["beams"] + 1, **i32)}
    arr = (_lib.SuffixReq * max(len(recs), 1))(*[_lib.SuffixReq(*r) for r in recs])
    host = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
    dev_recs = host.to(device)
    lib = _lib.load()
    stream = torch.cuda.current_stream(device).cuda_stream
    rc = lib.gr_suffix_metadata(dev_recs.data_ptr(), len(recs), tot["beams"], tot["prefix"], tot["suffix"],
                                out["mega_prefix_indices"].data_ptr(), out["suffix_slot_mapping_out"].data_ptr(),
                                out["suffix_cu_seqlens_q"].data_ptr(), out["suffix_cu_seqlens_k"].data_ptr(),
                                None if err is None else err.data_ptr(), ctypes.c_void_p(stream))
    if rc != _lib.GR_OK:
        raise RuntimeError(f"gr_suffix_metadata failed: {_lib.STATUS_NAMES.get(rc, rc)}")
    cu_k = out["suffix_cu_seqlens_k"]
    out["suffix_seq_lens"] = cu_k[1:] - cu_k[:-1]
    out.update(suffix_total_tokens=tot["suffix"], suffix_max_q_len=tot["max_q"], suffix_max_seq_len=tot["max_k"])
    out["_records"] = dev_recs   # keeps the records alive until the stream has read them
    return out
