"""Build the C-ABI shared library (sm_100a) in-tree.

    python -m vllm_gr_ehaleva_b200.build            # -> vllm_gr_ehaleva_b200/_gr_beam.so

The library is plain CUDA C++ with an extern "C" interface (include/gr_beam.h);
it links the CUDA runtime statically and has no PyTorch dependency.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_NAME = "_gr_beam.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
SOURCES = ["gr_beam_step.cu", "gr_suffix_kv.cu", "gr_remux.cu"]
HEADERS = ["gr_device.cuh", "gr_step_ws.cuh", "gr_step_select_ws.cuh", "gr_nvtx.h"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = os.path.join(home, "bin", "nvcc")
    if os.path.exists(p):
        return p
    raise RuntimeError("nvcc not found (set CUDA_HOME)")


def _inputs():
    files = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    files.append(os.path.join(ROOT, "include", "gr_beam.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _inputs() if os.path.exists(f))


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    if not force and up_to_date():
        return LIB_PATH
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
           "-shared", "-I", os.path.join(ROOT, "include"), "-o", LIB_PATH + ".tmp"]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += list(extra_flags or [])
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
