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
