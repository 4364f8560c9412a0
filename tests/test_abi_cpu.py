"""C ABI on the CPU: the library loads without a GPU, exports every function
the header declares, its structs have the header's layout, and descriptor
validation answers without touching a device."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from vllm_gr_ehaleva_b200 import _lib
from vllm_gr_ehaleva_b200.sample.beam_search_sampler import make_desc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gr_beam.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int32_t|const char\*)\s+(gr_\w+)\s*\(", text, re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 8
    for n in names:
        assert hasattr(lib, n), f"{n} declared in gr_beam.h but not exported"
    assert set(_lib.EXPORTED_SYMBOLS) == set(names)
    assert lib.gr_abi_version() == 2
    assert lib.gr_status_string(-6) == b"GR_ERR_UNSUPPORTED"


def test_struct_layout_matches_header():
    src = r'''
#include <stdio.h>
#include <stddef.h>
#include "gr_beam.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu %zu\n", sizeof(gr_step_desc), sizeof(gr_step_io),
         offsetof(gr_step_desc, row_stride), offsetof(gr_step_desc, num_edges),
         offsetof(gr_step_desc, vocab_stride), offsetof(gr_step_io, cand_score), offsetof(gr_step_io, err));
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        got = list(map(int, subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()))
    want = [ctypes.sizeof(_lib.StepDesc), ctypes.sizeof(_lib.StepIO), _lib.StepDesc.row_stride.offset,
            _lib.StepDesc.num_edges.offset, _lib.StepDesc.vocab_stride.offset, _lib.StepIO.cand_score.offset,
            _lib.StepIO.err.offset]
    assert got == want


def _desc(**kw):
    base = dict(R=2, NB=4, B=4, V=1000, VL=1000, voff=0, row_stride=1000, dtype=1, mode=0, K=0, eos=-1, T=0, N=0, E=0)
    base.update(kw)
    return make_desc(**base)


@pytest.mark.parametrize("kw,status", [
    (dict(), 0),
    (dict(R=0), -2), (dict(NB=0), -2), (dict(B=0), -2),
    (dict(VL=1001), -2), (dict(voff=10), -2), (dict(row_stride=999), -2),
    (dict(dtype=7), -3), (dict(mode=3), -3),
    (dict(K=2000), -2), (dict(eos=1000), -2),
    (dict(VL=100, voff=3, VS=10), 0),             # strided shard: tokens 3, 13, ..., 993
    (dict(VL=101, voff=3, VS=10), -2),            # its last token 1003 is outside the vocabulary
    (dict(VS=-1), -2),
    (dict(B=3000), -6),                           # 2B beyond the shared-memory key list
    (dict(NB=100000, V=100000, VL=100000, row_stride=100000), -6),   # flat index beyond 32 bits
])
def test_workspace_size_validation(kw, status):
    lib = _lib.load()
    n = ctypes.c_size_t(0)
    assert lib.gr_beam_step_workspace_size(ctypes.byref(_desc(**kw)), ctypes.byref(n)) == status
    if status == 0:
        # tau [R] + row counts [R*NB] + row slots [R*NB][2B] (128-byte aligned pieces)
        assert n.value >= 2 * 8 + 2 * 4 * 4 + 2 * 4 * 8 * 8


def test_step_flags_validated_without_a_device():
    lib = _lib.load()
    n = ctypes.c_size_t(0)
    d = _desc()
    d.flags = _lib.GR_STEP_CLEAR_ERR
    assert lib.gr_beam_step_workspace_size(ctypes.byref(d), ctypes.byref(n)) == 0
    d.flags = 0x2                                   # no such flag
    assert lib.gr_beam_step_workspace_size(ctypes.byref(d), ctypes.byref(n)) == -2
    # the vocab-sharded calls share one error word across three calls: no flags there
    d.flags = _lib.GR_STEP_CLEAR_ERR
    io = _lib.StepIO()
    part = ctypes.c_float(0.0)
    assert lib.gr_lse_partials(ctypes.byref(d), ctypes.byref(io), ctypes.byref(part), None, 0, None) == -2
    keys = ctypes.c_uint64(0)
    assert lib.gr_shard_candidates(ctypes.byref(d), ctypes.byref(io), ctypes.byref(part), 2, ctypes.byref(keys),
                                   None, 0, None) == -2
    assert lib.gr_merge_candidates(ctypes.byref(d), ctypes.byref(io), ctypes.byref(keys), 2, None, 0, None) == -2


def test_null_arguments_rejected_before_any_device_work():
    lib = _lib.load()
    d = _desc()
    io = _lib.StepIO()
    assert lib.gr_beam_step(None, ctypes.byref(io), None, 0, None) == -1
    assert lib.gr_beam_step(ctypes.byref(d), ctypes.byref(io), None, 0, None) == -1   # logits missing
    assert lib.gr_beam_step_noalloc(None, None, None) == -1


def test_sampler_refuses_to_run_without_the_library(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(ImportError):
        _lib.load(str(tmp_path / "missing.so"))


def test_attention_and_worker_struct_layouts_match_header():
    src = r'''
#include <stdio.h>
#include <stddef.h>
#include "gr_beam.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu %zu %zu\n", sizeof(gr_kv_gather_desc), offsetof(gr_kv_gather_desc, k_stride_tok),
         sizeof(gr_suffix_req), offsetof(gr_suffix_req, beam_base), offsetof(gr_suffix_req, own_total),
         sizeof(gr_remux_desc), offsetof(gr_remux_desc, max_dim), offsetof(gr_remux_desc, ids_bytes));
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        got = list(map(int, subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()))
    want = [ctypes.sizeof(_lib.KvGatherDesc), _lib.KvGatherDesc.k_stride_tok.offset, ctypes.sizeof(_lib.SuffixReq),
            _lib.SuffixReq.beam_base.offset, _lib.SuffixReq.own_total.offset, ctypes.sizeof(_lib.RemuxDesc),
            _lib.RemuxDesc.max_dim.offset, _lib.RemuxDesc.ids_bytes.offset]
    assert got == want


def test_attention_and_worker_entry_points_validate_without_a_device():
    # every case below returns before any CUDA call
    lib = _lib.load()
    g = _lib.KvGatherDesc(num_out=0, num_src=1, num_slots=1, num_heads=1, head_dim=8, elem_bytes=2)
    assert lib.gr_suffix_kv_gather(None, None, None, None, None, None, None, None, None) == -1
    assert lib.gr_suffix_kv_gather(ctypes.byref(g), None, None, None, None, None, None, None, None) == 0
    g.elem_bytes = 3
    assert lib.gr_suffix_kv_gather(ctypes.byref(g), None, None, None, None, None, None, None, None) == -3
    g.elem_bytes, g.num_heads = 2, 0
    assert lib.gr_suffix_kv_gather(ctypes.byref(g), None, None, None, None, None, None, None, None) == -2
    # metadata: sizes negative or records without beams / beams without records
    assert lib.gr_suffix_metadata(None, 0, 0, 0, -1, None, None, None, None, None, None) == -2
    out = (ctypes.c_int32 * 2)()
    assert lib.gr_suffix_metadata(None, 1, 0, 0, 0, None, None, out, out, None, None) == -2
    assert lib.gr_suffix_metadata(None, 0, 0, 0, 0, None, None, None, None, None, None) == -1
    # remux: K must be positive, integer widths 0/4/8, st 4/8; no request -> nothing to do
    r = _lib.RemuxDesc(num_requests=0, K=4, max_dim=8, num_rows=0, st_bytes=4)
    assert lib.gr_remux_logprobs(ctypes.byref(r), *([None] * 10), None) == 0
    r.K = 0
    assert lib.gr_remux_logprobs(ctypes.byref(r), *([None] * 10), None) == -2
    r.K, r.ids_bytes = 4, 2
    assert lib.gr_remux_logprobs(ctypes.byref(r), *([None] * 10), None) == -3


def test_a_c_program_links_against_the_library():
    # what a C or C++ caller does: include the header, link the shared library, call it
    src = r'''
#include <stdio.h>
#include "gr_beam.h"
int main(void) {
  gr_step_desc d = {0};
  d.num_requests = 2; d.num_beams = 4; d.beam_width = 4; d.vocab_size = 1000; d.vocab_local = 1000;
  d.row_stride = 1000; d.logit_dtype = GR_DTYPE_BF16; d.logprobs_mode = GR_LOGPROBS_RAW; d.eos_token_id = -1;
  size_t n = 0;
  int st = gr_beam_step_workspace_size(&d, &n);
  d.beam_width = 0;
  int bad = gr_beam_step_workspace_size(&d, &n);
  printf("%d %d %s %d\n", st, bad, gr_status_string(bad), gr_abi_version());
  return (st == GR_OK && n > 0 && bad == GR_ERR_BAD_DESC) ? 0 : 1;
}
'''
    lib = _lib.LIB_PATH
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "caller.c")
        exe = os.path.join(d, "caller")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, lib, f"-Wl,-rpath,{os.path.dirname(lib)}",
                        "-o", exe], check=True)
        r = subprocess.run([exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.split() == ["0", "-2", "GR_ERR_BAD_DESC", "2"]
