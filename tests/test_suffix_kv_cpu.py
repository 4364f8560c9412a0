"""Suffix KV pass on the CPU: the oracle's restatement of the reference's
metadata builder against the reference's own outputs (golden), the oracle
gather against a direct loop, and the wrapper's argument checks."""
import json
import os

import numpy as np
import pytest

from oracle import suffix_kv as osk

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "suffix_metadata.json")


def _cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


def _q_starts(c):
    per = c["beam_width"] * c["q_seq_len"]
    return list(range(0, per * c["batch_size"] + 1, per))


@pytest.mark.parametrize("idx", range(len(_cases())))
def test_metadata_matches_reference(idx):
    c = _cases()[idx]
    mega = [dict(prefix_len=c["prefix_len"], cache_len=0, beam_width=c["beam_width"], steps=c["suffix_kv_len"])
            ] * c["batch_size"]
    pi, smo, q_lens, seq_lens = osk.suffix_metadata(mega, _q_starts(c), c["block_size"])
    assert len(smo) == c["suffix_total_tokens"]
    if c["suffix_total_tokens"] == 0:
        assert c["suffix_slot_mapping_out"] is None or len(c["suffix_slot_mapping_out"]) == 0
        return
    np.testing.assert_array_equal(pi, np.asarray(c["mega_prefix_indices"]))
    np.testing.assert_array_equal(smo, np.asarray(c["suffix_slot_mapping_out"]))
    np.testing.assert_array_equal(seq_lens, np.asarray(c["suffix_seq_lens"]))
    np.testing.assert_array_equal(np.concatenate([[0], np.cumsum(seq_lens)]), np.asarray(c["suffix_cu_seqlens_k"]))
    np.testing.assert_array_equal(np.concatenate([[0], np.cumsum(q_lens)]), np.asarray(c["suffix_cu_seqlens_q"]))


def test_oracle_gather_matches_loop():
    rng = np.random.default_rng(0)
    nb, bs, H, D = 5, 16, 3, 8
    k = rng.standard_normal((nb, bs, H, D)).astype(np.float32)
    v = rng.standard_normal((nb, bs, H, D)).astype(np.float32)
    sm = rng.permutation(nb * bs)[:40].astype(np.int64)
    smo = rng.integers(0, 40, 70).astype(np.int32)
    ok, ov = osk.gather(k, v, sm, smo, 70)
    for t in range(70):
        s = sm[smo[t]]
        np.testing.assert_array_equal(ok[t], k[s // bs, s % bs])
        np.testing.assert_array_equal(ov[t], v[s // bs, s % bs])


def test_wrapper_rejects_bad_arguments():
    torch = pytest.importorskip("torch")
    from vllm_gr_ehaleva_b200.attention import suffix_kv
    k = torch.zeros(2, 16, 2, 64, dtype=torch.bfloat16)
    sm = torch.zeros(4, dtype=torch.long)
    smo = torch.zeros(3, dtype=torch.int32)
    with pytest.raises(ValueError):
        suffix_kv.gather_desc(k, k, sm, smo, 4)           # more output tokens than mapping entries
    with pytest.raises(ValueError):
        suffix_kv.gather_desc(k, k.float(), sm, smo, 3)   # K and V dtypes differ
    d = suffix_kv.gather_desc(k, k, sm, smo, 3)
    assert (d.num_out, d.num_src, d.num_slots, d.num_heads, d.head_dim, d.elem_bytes) == (3, 4, 32, 2, 64, 2)
    assert (d.k_stride_tok, d.k_stride_head, d.k_stride_dim) == (128, 64, 1)
    # a K view of an interleaved K/V cache: the flat slot range stays inside the storage
    kv = torch.zeros(2, 2, 16, 2, 64, dtype=torch.bfloat16)
    d = suffix_kv.gather_desc(kv[:, 0], kv[:, 1], sm, smo, 3)
    assert d.k_stride_tok == 128 and d.num_slots <= 2 * 16


def _expand(recs, tot):
    """The arrays gr_suffix_metadata writes, from its records (the formulas of
    its declaration in include/gr_beam.h), in NumPy."""
    pi = np.zeros(tot["prefix"], np.int64)
    smo = np.zeros(tot["suffix"], np.int32)
    cu_q = np.zeros(tot["beams"] + 1, np.int32)
    cu_k = np.zeros(tot["beams"] + 1, np.int32)
    for (q_start, out_base, suffix_base, beam_base, beams, remaining, steps, own0, own_total) in recs:
        pi[out_base:out_base + own_total] = q_start + np.arange(own_total)
        k = suffix_base
        q = out_base
        for b in range(beams):
            own = own0 if b == 0 else min(steps, own_total - own0 - (b - 1) * steps)
            if b == 0:
                vals = out_base + np.arange(own0)
            else:
                vals = np.concatenate([out_base + np.arange(remaining),
                                       out_base + own0 + (b - 1) * steps + np.arange(own)])
            smo[k:k + len(vals)] = vals
            k += len(vals)
            q += own
            cu_q[beam_base + b + 1] = q
            cu_k[beam_base + b + 1] = k
    return pi, smo, cu_q, cu_k


@pytest.mark.parametrize("idx", range(len(_cases())))
def test_device_metadata_records_match_reference(idx):
    from vllm_gr_ehaleva_b200.attention import suffix_records
    c = _cases()[idx]
    mega = [dict(prefix_len=c["prefix_len"], cache_len=0, beam_width=c["beam_width"], steps=c["suffix_kv_len"])
            ] * c["batch_size"]
    recs, tot = suffix_records(mega, _q_starts(c), c["block_size"])
    assert tot["suffix"] == c["suffix_total_tokens"]
    if tot["suffix"] == 0:
        return
    pi, smo, cu_q, cu_k = _expand(recs, tot)
    np.testing.assert_array_equal(pi, np.asarray(c["mega_prefix_indices"]))
    np.testing.assert_array_equal(smo, np.asarray(c["suffix_slot_mapping_out"]))
    np.testing.assert_array_equal(cu_q, np.asarray(c["suffix_cu_seqlens_q"]))
    np.testing.assert_array_equal(cu_k, np.asarray(c["suffix_cu_seqlens_k"]))
    assert tot["max_k"] == max(c["suffix_seq_lens"])


def test_records_mixed_requests_match_oracle():
    # standard requests between mega ones, a long uncached prefix, budgets that cut beams short
    from vllm_gr_ehaleva_b200.attention import suffix_records
    rng = np.random.default_rng(5)
    for _ in range(40):
        n = int(rng.integers(1, 7))
        q_lens = rng.integers(0, 200, n)
        q_starts = [0] + np.cumsum(q_lens).tolist()
        mega = []
        for i in range(n):
            if rng.random() < 0.25:
                mega.append(None)
                continue
            prefix = int(rng.integers(0, 80))
            mega.append(dict(prefix_len=prefix, cache_len=int(rng.integers(0, prefix + 1)),
                             beam_width=int(rng.integers(0, 9)), steps=int(rng.integers(0, 6))))
        block = int(rng.choice([16, 32]))
        pi, smo, q_l, seq_l = osk.suffix_metadata(mega, q_starts, block)
        recs, tot = suffix_records(mega, q_starts, block)
        e_pi, e_smo, e_cq, e_ck = _expand(recs, tot)
        np.testing.assert_array_equal(e_pi, pi)
        np.testing.assert_array_equal(e_smo, smo)
        np.testing.assert_array_equal(np.diff(e_cq), q_l)
        np.testing.assert_array_equal(np.diff(e_ck), seq_l)
        assert tot["max_q"] == (max(q_l) if len(q_l) else 0) and tot["max_k"] == (max(seq_l) if len(seq_l) else 0)


def _c_records(mega, q_starts, block):
    """gr_suffix_records through ctypes (host only)."""
    import ctypes
    from vllm_gr_ehaleva_b200 import _lib
    lib = _lib.load()
    n = len(q_starts) - 1
    flags = np.array([1 if m else 0 for m in mega], np.uint8)
    get = lambda k: np.array([int(m[k]) if m else 0 for m in mega], np.int32)  # noqa: E731
    arrs = [np.asarray(q_starts, np.int64), flags, get("prefix_len"), get("cache_len"), get("beam_width"),
            get("steps")]
    recs = (_lib.SuffixReq * max(n, 1))()
    totals = np.zeros(6, np.int64)
    rc = lib.gr_suffix_records(n, *[a.ctypes.data for a in arrs], block, ctypes.addressof(recs), totals.ctypes.data)
    assert rc == 0
    out = [(r.q_start, r.out_base, r.suffix_base, r.beam_base, r.beams, r.remaining, r.steps, r.own0, r.own_total)
           for r in recs[:int(totals[0])]]
    return out, dict(beams=int(totals[1]), prefix=int(totals[2]), suffix=int(totals[3]), max_q=int(totals[4]),
                     max_k=int(totals[5]))


def test_c_records_equal_python_records():
    from vllm_gr_ehaleva_b200.attention import suffix_records
    rng = np.random.default_rng(8)
    for _ in range(60):
        n = int(rng.integers(0, 9))
        q_starts = [0] + np.cumsum(rng.integers(0, 300, n)).tolist()
        mega = []
        for _i in range(n):
            if rng.random() < 0.25:
                mega.append(None)
                continue
            p = int(rng.integers(0, 90))
            mega.append(dict(prefix_len=p, cache_len=int(rng.integers(0, p + 1)), beam_width=int(rng.integers(0, 17)),
                             steps=int(rng.integers(0, 7))))
        block = int(rng.choice([16, 32]))
        assert _c_records(mega, q_starts, block) == suffix_records(mega, q_starts, block)
    for c in _cases():
        mega = [dict(prefix_len=c["prefix_len"], cache_len=0, beam_width=c["beam_width"],
                     steps=c["suffix_kv_len"])] * c["batch_size"]
        assert _c_records(mega, _q_starts(c), c["block_size"]) == suffix_records(mega, _q_starts(c), c["block_size"])


def test_c_records_refuse_fields_beyond_32_bits():
    # a request whose query tokens (and beams) do not fit the record's 32-bit
    # fields is refused, not wrapped: 2^32 query tokens, 2^31 - 1 beams of one step
    import ctypes
    from vllm_gr_ehaleva_b200 import _lib
    lib = _lib.load()
    q_starts = np.array([0, 2**32], np.int64)
    flags = np.array([1], np.uint8)
    plen, clen = np.array([10], np.int32), np.array([0], np.int32)
    w, st = np.array([2**31 - 1], np.int32), np.array([1], np.int32)
    recs = (_lib.SuffixReq * 1)()
    totals = np.zeros(6, np.int64)
    rc = lib.gr_suffix_records(1, q_starts.ctypes.data, flags.ctypes.data, plen.ctypes.data, clen.ctypes.data,
                               w.ctypes.data, st.ctypes.data, 16, ctypes.addressof(recs), totals.ctypes.data)
    assert rc == -2, _lib.STATUS_NAMES.get(rc, rc)     # GR_ERR_BAD_DESC
