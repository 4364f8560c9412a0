"""GPU parity of the suffix KV gather (gr_suffix_kv_gather) against the
reference's semantics (vllm_gr/v1/attention/backends/beam_attn.py:62-117):
bit-exact rows, on the reference builder's own suffix metadata for the
layouts of its cascade-attention test, on strided caches, on every element
size, and with out-of-range indices."""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from oracle import suffix_kv as osk  # noqa: E402
from vllm_gr_ehaleva_b200 import _lib  # noqa: E402
from vllm_gr_ehaleva_b200.attention import extract_suffix_kv  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "suffix_metadata.json")
DEV = "cuda"


def _golden():
    with open(GOLDEN) as f:
        return [c for c in json.load(f)["cases"] if c["suffix_total_tokens"] > 0]


def _expected(k_cache, v_cache, sm, smo, n):
    """The reference's addressing in torch: flat slot * stride(1)."""
    H, D = k_cache.shape[2], k_cache.shape[3]

    def flat(c):
        ns = c.shape[0] * c.shape[1]
        return c.as_strided((ns, H, D), (c.stride(1), c.stride(2), c.stride(3)))

    slots = sm.long()[smo[:n].long()]
    return flat(k_cache)[slots], flat(v_cache)[slots]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("heads,dim", [(4, 128), (2, 256)])
def test_reference_metadata_layouts(dtype, heads, dim):
    g = torch.Generator(device=DEV).manual_seed(0)
    for c in _golden():
        nb, bs = c["num_blocks"], c["block_size"]
        k = torch.randn(nb, bs, heads, dim, device=DEV, dtype=torch.float32, generator=g).to(dtype)
        v = torch.randn(nb, bs, heads, dim, device=DEV, dtype=torch.float32, generator=g).to(dtype)
        sm_all = torch.tensor(c["slot_mapping"], dtype=torch.long, device=DEV)
        sel = sm_all[torch.tensor(c["mega_prefix_indices"], dtype=torch.long, device=DEV)]
        smo = torch.tensor(c["suffix_slot_mapping_out"], dtype=torch.int32, device=DEV)
        n = c["suffix_total_tokens"]
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        ok, ov = extract_suffix_kv(k, v, sel, smo, n, err=err)
        ek, ev = _expected(k, v, sel, smo, n)
        assert torch.equal(ok, ek) and torch.equal(ov, ev), c
        assert int(err.item()) == 0


def test_matches_oracle_small():
    rng = np.random.default_rng(1)
    nb, bs, H, D = 6, 16, 2, 64
    k = rng.standard_normal((nb, bs, H, D)).astype(np.float32)
    v = rng.standard_normal((nb, bs, H, D)).astype(np.float32)
    sm = rng.permutation(nb * bs)[:50].astype(np.int64)
    smo = rng.integers(0, 50, 77).astype(np.int32)
    ek, ev = osk.gather(k, v, sm, smo, 77)
    ok, ov = extract_suffix_kv(torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV),
                               torch.from_numpy(sm).to(DEV), torch.from_numpy(smo).to(DEV), 77)
    np.testing.assert_array_equal(ok.cpu().numpy(), ek)
    np.testing.assert_array_equal(ov.cpu().numpy(), ev)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.uint8])
def test_element_sizes_and_odd_rows(dtype):
    # rows of 16-byte multiples take the vector kernel, others the element kernel
    for heads, dim in [(8, 128), (1, 8), (3, 5), (1, 1)]:
        nb, bs = 7, 32
        if dtype == torch.uint8:
            k = torch.randint(0, 256, (nb, bs, heads, dim), dtype=torch.uint8, device=DEV)
            v = torch.randint(0, 256, (nb, bs, heads, dim), dtype=torch.uint8, device=DEV)
        else:
            k = torch.randn(nb, bs, heads, dim, device=DEV).to(dtype)
            v = torch.randn(nb, bs, heads, dim, device=DEV).to(dtype)
        sm = torch.randperm(nb * bs, device=DEV)[:100]
        smo = torch.randint(0, 100, (333,), dtype=torch.int32, device=DEV)
        ok, ov = extract_suffix_kv(k, v, sm, smo, 333)
        ek, ev = _expected(k, v, sm, smo, 333)
        assert torch.equal(ok, ek) and torch.equal(ov, ev), (heads, dim)


def test_strided_caches():
    # K and V views of one interleaved cache (block stride = 2 x block_size rows),
    # the reference's flat-slot addressing applied as it does
    nb, bs, H, D = 9, 16, 4, 64
    kv = torch.randn(nb, 2, bs, H, D, device=DEV).to(torch.bfloat16)
    k, v = kv[:, 0], kv[:, 1]
    sm = torch.randperm(nb * bs, device=DEV)[:80]
    smo = torch.randint(0, 80, (500,), dtype=torch.int32, device=DEV)
    ok, ov = extract_suffix_kv(k, v, sm, smo, 500)
    ek, ev = _expected(k, v, sm, smo, 500)
    assert torch.equal(ok, ek) and torch.equal(ov, ev)
    # heads not adjacent to each other (element kernel with strides)
    base = torch.randn(nb, bs, D, H, device=DEV).to(torch.float16)
    k2 = base.transpose(2, 3)
    v2 = (base * 2).transpose(2, 3)
    ok, ov = extract_suffix_kv(k2, v2, sm, smo, 500)
    ek, ev = _expected(k2, v2, sm, smo, 500)
    assert torch.equal(ok, ek) and torch.equal(ov, ev)


def test_fewer_outputs_than_mapping_and_empty():
    nb, bs, H, D = 4, 16, 2, 128
    k = torch.randn(nb, bs, H, D, device=DEV).to(torch.bfloat16)
    v = torch.randn(nb, bs, H, D, device=DEV).to(torch.bfloat16)
    sm = torch.arange(nb * bs, device=DEV)
    smo = torch.randint(0, nb * bs, (100,), dtype=torch.int32, device=DEV)
    ok, ov = extract_suffix_kv(k, v, sm, smo, 37)
    ek, ev = _expected(k, v, sm, smo, 37)
    assert ok.shape == (37, H, D) and torch.equal(ok, ek) and torch.equal(ov, ev)
    ok, ov = extract_suffix_kv(k, v, sm, smo, 0)
    assert ok.shape == (0, H, D) and ov.shape == (0, H, D)


@pytest.mark.parametrize("vector", [True, False])
def test_out_of_range_indices(vector):
    nb, bs, H = 4, 16, 2
    D = 128 if vector else 3
    k = torch.randn(nb, bs, H, D, device=DEV).to(torch.bfloat16)
    v = torch.randn(nb, bs, H, D, device=DEV).to(torch.bfloat16)
    sm = torch.arange(nb * bs, device=DEV)
    sm[5] = -1                 # padding slot
    sm[6] = nb * bs            # past the cache
    smo = torch.tensor([0, 5, 6, 7, -3, 64, 1], dtype=torch.int32, device=DEV)   # -3, 64: outside slot_mapping
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    ok, ov = extract_suffix_kv(k, v, sm, smo, 7, err=err)
    assert int(err.item()) & 0x20
    good = [0, 3, 6]
    bad = [1, 2, 4, 5]
    ek, ev = _expected(k, v, sm.clamp(0, nb * bs - 1), smo.clamp(0, nb * bs - 1), 7)
    assert torch.equal(ok[good], ek[good]) and torch.equal(ov[good], ev[good])
    assert not ok[bad].float().abs().sum().item() and not ov[bad].float().abs().sum().item()
    assert _lib.describe_deverr(int(err.item())) == "GR_DEVERR_BAD_SLOT"


def test_large_gather():
    # ~65k output tokens x 2 KB rows: many warps, the persistent loop's wrap
    nb, bs, H, D = 4096, 16, 8, 128
    k = torch.randn(nb, bs, H, D, device=DEV).to(torch.bfloat16)
    v = torch.randn(nb, bs, H, D, device=DEV).to(torch.bfloat16)
    sm = torch.randperm(nb * bs, device=DEV)
    smo = torch.randint(0, nb * bs, (65537,), dtype=torch.int32, device=DEV)
    ok, ov = extract_suffix_kv(k, v, sm, smo, 65537)
    ek, ev = _expected(k, v, sm, smo, 65537)
    assert torch.equal(ok, ek) and torch.equal(ov, ev)


def _q_starts(c):
    per = c["beam_width"] * c["q_seq_len"]
    return list(range(0, per * c["batch_size"] + 1, per))


def test_device_metadata_matches_reference_builder():
    from vllm_gr_ehaleva_b200.attention import build_suffix_metadata
    for c in _golden():
        mega = [dict(prefix_len=c["prefix_len"], cache_len=0, beam_width=c["beam_width"],
                     steps=c["suffix_kv_len"])] * c["batch_size"]
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        m = build_suffix_metadata(mega, _q_starts(c), c["block_size"], DEV, err=err)
        assert m["suffix_total_tokens"] == c["suffix_total_tokens"]
        assert m["mega_prefix_indices"].cpu().tolist() == c["mega_prefix_indices"]
        assert m["suffix_slot_mapping_out"].cpu().tolist() == c["suffix_slot_mapping_out"]
        assert m["suffix_cu_seqlens_q"].cpu().tolist() == c["suffix_cu_seqlens_q"]
        assert m["suffix_cu_seqlens_k"].cpu().tolist() == c["suffix_cu_seqlens_k"]
        assert m["suffix_seq_lens"].cpu().tolist() == c["suffix_seq_lens"]
        assert int(err.item()) == 0


def test_device_metadata_random_layouts_match_oracle():
    from vllm_gr_ehaleva_b200.attention import build_suffix_metadata
    rng = np.random.default_rng(9)
    for _ in range(30):
        n = int(rng.integers(1, 40))
        q_lens = rng.integers(0, 600, n)
        q_starts = [0] + np.cumsum(q_lens).tolist()
        mega = [None if rng.random() < 0.2 else
                dict(prefix_len=int(p), cache_len=int(rng.integers(0, p + 1)), beam_width=int(rng.integers(0, 65)),
                     steps=int(rng.integers(0, 9))) for p in rng.integers(0, 100, n)]
        block = int(rng.choice([16, 32]))
        pi, smo, q_l, seq_l = osk.suffix_metadata(mega, q_starts, block)
        m = build_suffix_metadata(mega, q_starts, block, DEV)
        np.testing.assert_array_equal(m["mega_prefix_indices"].cpu().numpy(), pi)
        np.testing.assert_array_equal(m["suffix_slot_mapping_out"].cpu().numpy(), smo)
        np.testing.assert_array_equal(np.diff(m["suffix_cu_seqlens_q"].cpu().numpy()), q_l)
        np.testing.assert_array_equal(m["suffix_seq_lens"].cpu().numpy(), seq_l)


def test_device_metadata_rejects_inconsistent_records():
    # a record that points past the outputs: its writes are dropped and flagged
    import ctypes
    lib = _lib.load()
    rec = (_lib.SuffixReq * 1)(_lib.SuffixReq(0, 50, 0, 0, 2, 3, 4, 7, 11))   # out_base 50 > 11 prefix entries
    recs = torch.frombuffer(bytearray(bytes(rec)), dtype=torch.uint8).to(DEV)
    pi = torch.full((11,), -7, dtype=torch.int64, device=DEV)
    smo = torch.full((17,), -7, dtype=torch.int32, device=DEV)
    cq = torch.full((3,), -7, dtype=torch.int32, device=DEV)
    ck = torch.full((3,), -7, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = lib.gr_suffix_metadata(recs.data_ptr(), 1, 2, 11, 17, pi.data_ptr(), smo.data_ptr(), cq.data_ptr(),
                                ck.data_ptr(), err.data_ptr(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) & 0x40
    assert (pi == -7).all() and (smo == -7).all()


def test_metadata_first_then_gather_in_a_fresh_process():
    # both entry points share one per-device record: the first call of either must set all of it
    import subprocess
    import sys
    code = r'''
import torch
from vllm_gr_ehaleva_b200.attention import build_suffix_metadata, extract_suffix_kv
m = build_suffix_metadata([dict(prefix_len=3, cache_len=0, beam_width=4, steps=2)], [0, 11], 16, "cuda")
k = torch.randn(2, 16, 2, 64, device="cuda").to(torch.bfloat16)
sm = torch.arange(32, device="cuda")
ok, ov = extract_suffix_kv(k, k, sm, m["suffix_slot_mapping_out"], m["suffix_total_tokens"])
torch.cuda.synchronize()
exp = k.view(-1, 2, 64)[sm[m["suffix_slot_mapping_out"].long()]]
assert torch.equal(ok, exp), "gather after metadata"
print("ok")
'''
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]
