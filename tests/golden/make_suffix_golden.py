"""Record the reference's suffix-pass metadata as golden vectors.

    python tests/golden/make_suffix_golden.py <reference checkout>

For the mega-decode layouts of the reference's own cascade-attention kernel
test (tests/kernels/attention/test_cascade_beam_flash_attn.py: CASES, batch
sizes, beam widths, block sizes; its perf case too), runs the reference's
BeamAttentionMetadataBuilder.build (vllm_gr/v1/attention/backends/
beam_attn.py:480-559, plain Python on the CPU via oracle/ref_shim.py) and
writes tests/golden/suffix_metadata.json: per case the inputs (block tables,
slot mapping as the test builds them) and the builder's mega prefix indices,
suffix slot_mapping_out, suffix sequence lengths and cumulative lengths.  The
suffix KV gather (beam_attn.py:62-117) consumes exactly these.  The fixture is
committed; the tests read only it.
"""
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_shim  # noqa: E402

# (q_seq_len, kv_seq_len, suffix_kv_len) of the reference test, plus its perf case
LAYOUTS = [(8, 32, 8), (8, 8, 8), (4, 64, 4), (4, 16, 4), (1, 16, 4), (1, 128, 1), (4, 32, 7), (8, 2048, 8)]


def test_inputs(batch_size, beam_width, q_seq_len, kv_seq_len, suffix_kv_len, block_size):
    """Block tables and slot mapping as the reference test's prepare_inputs
    builds them (test_cascade_beam_flash_attn.py:92-170)."""
    shared = kv_seq_len - suffix_kv_len
    mega_seq_len = shared + beam_width * suffix_kv_len
    blocks_per_req = (mega_seq_len + block_size - 1) // block_size
    block_tables = torch.stack([torch.arange(i * blocks_per_req, (i + 1) * blocks_per_req, dtype=torch.int32)
                                for i in range(batch_size)])
    num_actual = batch_size * beam_width * q_seq_len
    slot_mapping = torch.zeros(num_actual, dtype=torch.long)
    budget = beam_width * q_seq_len
    cache_len = (shared // block_size) * block_size
    write_len = min(shared - cache_len + beam_width * suffix_kv_len, budget)
    for i in range(batch_size):
        phys = (block_tables[i].to(torch.long).unsqueeze(-1) * block_size + torch.arange(block_size)).view(-1)
        slot_mapping[i * budget: i * budget + write_len] = phys[cache_len: cache_len + write_len]
    return shared, block_tables, slot_mapping, batch_size * blocks_per_req


def main(reference_root):
    cases = []
    for (q, kv, sfx) in LAYOUTS:
        batches = [8] if kv == 2048 else [1, 4]
        beams = [16, 32, 128] if kv == 2048 else [16, 32]
        for bs in batches:
            for bw in beams:
                for block in (16, 32):
                    shared, bt, sm, nblocks = test_inputs(bs, bw, q, kv, sfx, block)
                    meta = ref_shim.reference_suffix_metadata(
                        reference_root, num_reqs=bs, beam_width=bw, q_seq_len=q, prefix_len=shared, steps=sfx,
                        cache_len=0, block_size=block, block_tables=bt, slot_mapping=sm)
                    cases.append(dict(batch_size=bs, beam_width=bw, q_seq_len=q, kv_seq_len=kv, suffix_kv_len=sfx,
                                      block_size=block, num_blocks=nblocks, prefix_len=shared,
                                      slot_mapping=sm.tolist(), **meta))
    out = os.path.join(HERE, "suffix_metadata.json")
    with open(out, "w") as f:
        json.dump({"source": "vllm_gr/v1/attention/backends/beam_attn.py:255-413, 432-559 (reference builder)",
                   "cases": cases}, f, separators=(",", ":"))
    print(f"wrote {out}: {len(cases)} cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GR_REFERENCE_ROOT", ""))
