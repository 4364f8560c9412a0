"""ctypes binding of the C ABI in include/gr_beam.h.

The shared library is the product path; there is no fallback.  If it is not
built, importing the sampler raises ImportError with the build command.
"""
from __future__ import annotations

import ctypes
import os

from .build import LIB_PATH

GR_OK = 0
GR_STEP_CLEAR_ERR = 0x1      # gr_step_desc.flags: the step zeroes io->err itself
STATUS_NAMES = {
    0: "GR_OK", -1: "GR_ERR_NULL", -2: "GR_ERR_BAD_DESC", -3: "GR_ERR_DTYPE",
    -4: "GR_ERR_MISALIGNED", -5: "GR_ERR_WORKSPACE", -6: "GR_ERR_UNSUPPORTED",
    -7: "GR_ERR_CUDA", -8: "GR_ERR_NO_DEVICE",
}
DEVERR_NAMES = {
    0x1: "GR_DEVERR_BAD_NODE", 0x2: "GR_DEVERR_BAD_CHILD", 0x4: "GR_DEVERR_TIMEOUT",
    0x8: "GR_DEVERR_OVERFLOW", 0x10: "GR_DEVERR_TIE_BOUNDARY", 0x20: "GR_DEVERR_BAD_SLOT",
    0x40: "GR_DEVERR_BAD_RECORD",
}
DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
LOGPROBS_RAW, LOGPROBS_PROCESSED = 0, 1
NODE_UNCONSTRAINED, NODE_DEAD = -1, -2

EXPORTED_SYMBOLS = (
    "gr_abi_version", "gr_status_string", "gr_beam_step_workspace_size", "gr_beam_step",
    "gr_lse_partials", "gr_shard_candidates", "gr_merge_candidates", "gr_beam_step_noalloc",
    "gr_suffix_kv_gather", "gr_suffix_metadata", "gr_suffix_records", "gr_remux_logprobs",
)
NOALLOC_SCRATCH_BYTES = 16 << 20


class StepDesc(ctypes.Structure):
    _fields_ = [
        ("num_requests", ctypes.c_int32),
        ("num_beams", ctypes.c_int32),
        ("beam_width", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32),
        ("vocab_local", ctypes.c_int32),
        ("vocab_offset", ctypes.c_int32),
        ("row_stride", ctypes.c_int64),
        ("logit_dtype", ctypes.c_int32),
        ("logprobs_mode", ctypes.c_int32),
        ("per_beam_k", ctypes.c_int32),
        ("eos_token_id", ctypes.c_int32),
        ("hist_len", ctypes.c_int32),
        ("num_nodes", ctypes.c_int32),
        ("num_edges", ctypes.c_int64),
        ("vocab_stride", ctypes.c_int32),
        ("flags", ctypes.c_int32),
    ]


_IO_FIELDS = (
    "logits", "cum", "node", "row_ptr", "child_tok", "child_node", "temperature", "rep_penalty",
    "pres_penalty", "freq_penalty", "hist_in", "cand_score", "cand_token", "cand_parent",
    "sel_score", "sel_token", "sel_parent", "sel_node", "eos_score", "hist_out", "lse", "err",
)


class StepIO(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in _IO_FIELDS]


class SuffixReq(ctypes.Structure):
    _fields_ = [
        ("q_start", ctypes.c_int64),
        ("out_base", ctypes.c_int64),
        ("suffix_base", ctypes.c_int64),
        ("beam_base", ctypes.c_int32),
        ("beams", ctypes.c_int32),
        ("remaining", ctypes.c_int32),
        ("steps", ctypes.c_int32),
        ("own0", ctypes.c_int32),
        ("own_total", ctypes.c_int32),
    ]


class RemuxDesc(ctypes.Structure):
    _fields_ = [
        ("num_requests", ctypes.c_int32),
        ("K", ctypes.c_int32),
        ("max_dim", ctypes.c_int64),
        ("num_rows", ctypes.c_int64),
        ("lps_stride", ctypes.c_int64),
        ("ids_stride", ctypes.c_int64),
        ("st_stride", ctypes.c_int64),
        ("ids_bytes", ctypes.c_int32),
        ("ranks_bytes", ctypes.c_int32),
        ("st_bytes", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class KvGatherDesc(ctypes.Structure):
    _fields_ = [
        ("num_out", ctypes.c_int64),
        ("num_src", ctypes.c_int64),
        ("num_slots", ctypes.c_int64),
        ("num_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("elem_bytes", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("k_stride_tok", ctypes.c_int64),
        ("k_stride_head", ctypes.c_int64),
        ("k_stride_dim", ctypes.c_int64),
        ("v_stride_tok", ctypes.c_int64),
        ("v_stride_head", ctypes.c_int64),
        ("v_stride_dim", ctypes.c_int64),
    ]


def describe_deverr(code: int) -> str:
    names = [n for bit, n in DEVERR_NAMES.items() if code & bit]
    return "|".join(names) if names else "0"


_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load the library (once).  Raises ImportError if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m vllm_gr_ehaleva_b200.build`")
    lib = ctypes.CDLL(path)
    P = ctypes.POINTER
    lib.gr_abi_version.restype = ctypes.c_int32
    lib.gr_abi_version.argtypes = []
    lib.gr_status_string.restype = ctypes.c_char_p
    lib.gr_status_string.argtypes = [ctypes.c_int32]
    lib.gr_beam_step_workspace_size.restype = ctypes.c_int32
    lib.gr_beam_step_workspace_size.argtypes = [P(StepDesc), P(ctypes.c_size_t)]
    lib.gr_beam_step.restype = ctypes.c_int32
    lib.gr_beam_step.argtypes = [P(StepDesc), P(StepIO), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.gr_beam_step_noalloc.restype = ctypes.c_int32
    lib.gr_beam_step_noalloc.argtypes = [P(StepDesc), P(StepIO), ctypes.c_void_p]
    lib.gr_lse_partials.restype = ctypes.c_int32
    lib.gr_lse_partials.argtypes = [P(StepDesc), P(StepIO), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                    ctypes.c_void_p]
    lib.gr_shard_candidates.restype = ctypes.c_int32
    lib.gr_shard_candidates.argtypes = [P(StepDesc), P(StepIO), ctypes.c_void_p, ctypes.c_int32,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.gr_merge_candidates.restype = ctypes.c_int32
    lib.gr_merge_candidates.argtypes = [P(StepDesc), P(StepIO), ctypes.c_void_p, ctypes.c_int32,
                                        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.gr_suffix_kv_gather.restype = ctypes.c_int32
    lib.gr_suffix_kv_gather.argtypes = [P(KvGatherDesc), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p]
    lib.gr_suffix_metadata.restype = ctypes.c_int32
    lib.gr_suffix_metadata.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.gr_suffix_records.restype = ctypes.c_int32
    lib.gr_suffix_records.argtypes = [ctypes.c_int32] + [ctypes.c_void_p] * 6 + [ctypes.c_int32, ctypes.c_void_p,
                                                                                ctypes.c_void_p]
    lib.gr_remux_logprobs.restype = ctypes.c_int32
    lib.gr_remux_logprobs.argtypes = [P(RemuxDesc)] + [ctypes.c_void_p] * 11
    _lib = lib
    return lib


def check(status: int, what: str = "gr call") -> None:
    if status != GR_OK:
        raise RuntimeError(f"{what} failed: {STATUS_NAMES.get(status, status)}")
