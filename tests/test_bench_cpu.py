"""Host logic of bench.py: how requests split over ranks, which kernels a
workload launches (the line's gpu_launches and kernel name), and the
algorithmic bytes the roofline divides by."""
import numpy as np
import pytest

import bench
from vllm_gr_ehaleva_b200.synthetic import CONFIGS


def _wl(cfg_name, R=2, catalog=None):
    c = CONFIGS[cfg_name]
    return dict(cfg=c, R=R, B=c["beams"], V=c["vocab"], catalog=catalog)


def test_requests_per_rank():
    assert bench.requests_per_rank("cfg2", None, 8) == CONFIGS["cfg2"]["requests"]   # weak: per rank
    assert bench.requests_per_rank("cfg3", None, 4) == CONFIGS["cfg3"]["requests"] // 4   # strong: split
    assert bench.requests_per_rank("cfg3", 5, 4) == 5                               # explicit override
    with pytest.raises(SystemExit):
        bench.requests_per_rank("cfg3", None, 3)                                    # 128 over 3 ranks


def test_kernel_names_and_launch_counts(monkeypatch):
    monkeypatch.delenv("GR_BEAM_KERNEL", raising=False)
    free = _wl("cfg4")                       # no catalog, processed with penalties
    assert bench.step_kernel_name(free) == "fused_select_ws_kernel"
    assert bench.pen_tables_launched(free)   # row_meta + pen_table + select + merge
    raw_free = _wl("cfg4")
    raw_free["cfg"] = dict(CONFIGS["cfg4"], mode="raw")
    assert not bench.pen_tables_launched(raw_free)
    monkeypatch.setenv("GR_BEAM_KERNEL", "stream")
    assert bench.step_kernel_name(free) == "fused_step_kernel"
    assert not bench.pen_tables_launched(free)


def test_algorithmic_bytes_of_a_step_without_a_catalog():
    wl = _wl("cfg4", R=2)
    B, V, T = wl["B"], wl["V"], 64
    got = bench.algorithmic_bytes(wl, np.full((2, B), -1, np.int32), T)
    want = 2 * (B * V * 4 + B * 12 + 2 * B * 12 + B * 16 + B * T * 4 + B * (T + 1) * 4 + B * T * 4)
    assert got == want
