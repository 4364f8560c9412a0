"""PyTorch front end of the device beam step.

This fills the slot the reference reserves for its beam-search sampler
(vllm_gr/sample/__init__.py:1-3, planned as sample/beam_search_sampler.py in
the reference's own design notes, section 3.6 "Sample").  One ``BeamSearchSampler.step`` call takes
the logits rows of all beams of all requests and returns what the reference's
per-step host code computes from vLLM's flat logprobs
(serving_engine.py:457-597 / llm.py:201-280):

    sel_parent / sel_token / sel_score   the new beams (fork_info + cum_logprob)
    sel_node                             their trie nodes (Catalog.valid state)
    hist_out                             forked per-beam token table
    eos_score                            per-beam EOS completion score (NaN: none)
    cand_*                               the canonical top-2B candidates

Tensors stay on the GPU; the step is stream ordered and does not synchronise.
PyTorch only allocates the buffers; the arithmetic is the CUDA library's.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from .. import _lib

LOGPROBS_MODES = {"raw_logprobs": _lib.LOGPROBS_RAW, "processed_logprobs": _lib.LOGPROBS_PROCESSED}
_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


@dataclass
class BeamStepOutput:
    cand_score: torch.Tensor
    cand_token: torch.Tensor
    cand_parent: torch.Tensor
    sel_score: torch.Tensor
    sel_token: torch.Tensor
    sel_parent: torch.Tensor
    sel_node: torch.Tensor
    eos_score: torch.Tensor
    hist_out: torch.Tensor
    lse: torch.Tensor
    err: torch.Tensor

    def check(self) -> None:
        """Synchronise and raise if the device reported an error."""
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"beam step device error: {_lib.describe_deverr(code)}")


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _per_request(v, R: int, device) -> Optional[torch.Tensor]:
    if v is None:
        return None
    if isinstance(v, torch.Tensor):
        t = v.to(device=device, dtype=torch.float32).reshape(-1)
    else:
        # host values go through pinned memory with an asynchronous copy: a
        # copy from pageable memory would make the host wait for the stream
        # (every step queued before this one) on every call
        t = torch.tensor([float(x) for x in (v if isinstance(v, Sequence) else [v] * R)], dtype=torch.float32)
        if torch.device(device).type == "cuda":
            t = t.pin_memory().to(device=device, non_blocking=True)
        else:
            t = t.to(device=device)
    if t.numel() == 1 and R > 1:
        t = t.expand(R).contiguous()
    if t.numel() != R:
        raise ValueError("per-request parameter must have one value per request")
    return t.contiguous()


class Workspace:
    """Grow-only device workspace (one per sampler / stream)."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.buf: Optional[torch.Tensor] = None

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.device)
        return self.buf


def make_desc(*, R, NB, B, V, VL, voff, row_stride, dtype, mode, K, eos, T, N, E, VS=1) -> _lib.StepDesc:
    d = _lib.StepDesc()
    d.num_requests, d.num_beams, d.beam_width = R, NB, B
    d.vocab_size, d.vocab_local, d.vocab_offset, d.vocab_stride = V, VL, voff, VS
    d.row_stride = row_stride
    d.logit_dtype, d.logprobs_mode, d.per_beam_k = dtype, mode, K
    d.eos_token_id, d.hist_len, d.num_nodes, d.num_edges = eos, T, N, E
    return d


def workspace_size(desc: _lib.StepDesc) -> int:
    lib = _lib.load()
    n = ctypes.c_size_t(0)
    _lib.check(lib.gr_beam_step_workspace_size(ctypes.byref(desc), ctypes.byref(n)), "gr_beam_step_workspace_size")
    return int(n.value)


def _prepare(logits: torch.Tensor, cum: torch.Tensor, node: torch.Tensor, *, beam_width: int,
             csr: Optional[tuple] = None, vocab_size: Optional[int] = None, vocab_offset: int = 0,
             logprobs_mode: str = "raw_logprobs", per_beam_k: int = 0, eos_token_id: Optional[int] = None,
             hist: Optional[torch.Tensor] = None, temperature=None, repetition_penalty=None,
             presence_penalty=None, frequency_penalty=None, workspace: Optional[Workspace] = None,
             stream: Optional[torch.cuda.Stream] = None, vocab_stride: int = 1, clear_err: bool = False):
    """Checks the step inputs and builds (descriptor, io, outputs, workspace, stream).
    Local logit column j holds token vocab_offset + j * vocab_stride.  clear_err
    (single-call steps): the library zeroes the error word itself
    (GR_STEP_CLEAR_ERR), so it is allocated without a fill."""
    if not logits.is_cuda:
        raise ValueError("logits must be a CUDA tensor")
    device = logits.device
    if cum.dim() != 2:
        raise ValueError("cum must be [R, num_beams]")
    R, NB = cum.shape
    if logits.dim() == 3:
        if logits.shape[0] != R or logits.shape[1] != NB:
            raise ValueError("logits must be [R, num_beams, V_l]")
        if logits.stride(2) != 1 or logits.stride(0) != NB * logits.stride(1):
            raise ValueError("logits rows must be evenly strided with unit column stride")
        VL, row_stride = logits.shape[2], logits.stride(1)
    elif logits.dim() == 2:
        if logits.shape[0] != R * NB or logits.stride(1) != 1:
            raise ValueError("logits must be [R*num_beams, V_l] with unit column stride")
        VL, row_stride = logits.shape[1], logits.stride(0)
    else:
        raise ValueError("logits must be 2-D or 3-D")
    if logits.dtype not in _DTYPES:
        raise ValueError(f"unsupported logits dtype {logits.dtype}")
    V = int(vocab_size if vocab_size is not None else VL)
    B = int(beam_width)
    cum = cum.to(device=device, dtype=torch.float32).contiguous()
    node = node.to(device=device, dtype=torch.int32).contiguous()
    if node.shape != (R, NB):
        raise ValueError("node must be [R, num_beams]")
    T = 0
    if hist is not None:
        if hist.dim() != 3 or hist.shape[0] != R or hist.shape[1] != NB:
            raise ValueError("hist must be [R, num_beams, T]")
        hist = hist.to(device=device, dtype=torch.int32).contiguous()
        T = hist.shape[2]
        if T == 0:
            hist = None
    if csr is not None:
        row_ptr, child_tok, child_node = csr
        N, E = int(row_ptr.numel()) - 1, int(child_tok.numel())
    else:
        row_ptr = child_tok = child_node = None
        N, E = 0, 0
    mode = LOGPROBS_MODES[logprobs_mode]
    eos = -1 if eos_token_id is None else int(eos_token_id)
    desc = make_desc(R=R, NB=NB, B=B, V=V, VL=VL, voff=int(vocab_offset), row_stride=int(row_stride),
                     dtype=_DTYPES[logits.dtype], mode=mode, K=int(per_beam_k), eos=eos, T=T, N=N, E=E,
                     VS=int(vocab_stride))
    if clear_err:
        desc.flags = _lib.GR_STEP_CLEAR_ERR
    temps = _per_request(temperature, R, device)
    reps = _per_request(repetition_penalty, R, device)
    press = _per_request(presence_penalty, R, device)
    freqs = _per_request(frequency_penalty, R, device)

    f32 = dict(dtype=torch.float32, device=device)
    i32 = dict(dtype=torch.int32, device=device)
    out = BeamStepOutput(
        cand_score=torch.empty((R, 2 * B), **f32), cand_token=torch.empty((R, 2 * B), **i32),
        cand_parent=torch.empty((R, 2 * B), **i32), sel_score=torch.empty((R, B), **f32),
        sel_token=torch.empty((R, B), **i32), sel_parent=torch.empty((R, B), **i32),
        sel_node=torch.empty((R, B), **i32), eos_score=torch.empty((R, NB), **f32),
        hist_out=torch.empty((R, B, T + 1), **i32), lse=torch.empty((R, NB), **f32),
        err=torch.empty(1, **i32) if clear_err else torch.zeros(1, **i32))
    io = _lib.StepIO()
    io.logits, io.cum, io.node = _ptr(logits), _ptr(cum), _ptr(node)
    io.row_ptr, io.child_tok, io.child_node = _ptr(row_ptr), _ptr(child_tok), _ptr(child_node)
    io.temperature, io.rep_penalty, io.pres_penalty, io.freq_penalty = _ptr(temps), _ptr(reps), _ptr(press), _ptr(freqs)
    io.hist_in = _ptr(hist)
    io.cand_score, io.cand_token, io.cand_parent = _ptr(out.cand_score), _ptr(out.cand_token), _ptr(out.cand_parent)
    io.sel_score, io.sel_token, io.sel_parent, io.sel_node = (_ptr(out.sel_score), _ptr(out.sel_token),
                                                               _ptr(out.sel_parent), _ptr(out.sel_node))
    io.eos_score, io.hist_out, io.lse, io.err = _ptr(out.eos_score), _ptr(out.hist_out), _ptr(out.lse), _ptr(out.err)
    nbytes = workspace_size(desc)
    ws = (workspace or Workspace(device)).get(nbytes)
    # the tensors the io pointers refer to stay alive with the returned tuple
    keep = (logits, cum, node, hist, row_ptr, child_tok, child_node, temps, reps, press, freqs)
    s = _launch_stream(stream, device, keep + tuple(vars(out).values()) + (ws,))
    return desc, io, out, ws, s, keep


def _launch_stream(stream: Optional[torch.cuda.Stream], device, tensors) -> torch.cuda.Stream:
    """The stream the library calls run on.  The inputs, their converted
    copies and the outputs were made on the current stream: a different
    launch stream first waits for the current one, and every tensor the call
    reads or writes is recorded as used on it, so that the caching allocator
    does not hand its memory out again before the call's kernels are done."""
    cur = torch.cuda.current_stream(device)
    if stream is None or stream == cur:
        return cur
    stream.wait_stream(cur)
    for t in tensors:
        if isinstance(t, torch.Tensor) and t.is_cuda:
            t.record_stream(stream)
    return stream


def beam_step(logits: torch.Tensor, cum: torch.Tensor, node: torch.Tensor, *, beam_width: int,
              csr: Optional[tuple] = None, vocab_size: Optional[int] = None, vocab_offset: int = 0,
              logprobs_mode: str = "raw_logprobs", per_beam_k: int = 0, eos_token_id: Optional[int] = None,
              hist: Optional[torch.Tensor] = None, temperature=None, repetition_penalty=None,
              presence_penalty=None, frequency_penalty=None, workspace: Optional[Workspace] = None,
              stream: Optional[torch.cuda.Stream] = None) -> BeamStepOutput:
    """One device beam step.  Shapes: logits [R, NB, V_l] (or [R*NB, V_l] with cum/node [R, NB]),
    cum float32 [R, NB], node int32 [R, NB], hist int32 [R, NB, T], csr = (row_ptr int64,
    child_tok int32, child_node int32) device tensors."""
    lib = _lib.load()
    desc, io, out, ws, s, _keep = _prepare(
        logits, cum, node, beam_width=beam_width, csr=csr, vocab_size=vocab_size, vocab_offset=vocab_offset,
        logprobs_mode=logprobs_mode, per_beam_k=per_beam_k, eos_token_id=eos_token_id, hist=hist,
        temperature=temperature, repetition_penalty=repetition_penalty, presence_penalty=presence_penalty,
        frequency_penalty=frequency_penalty, workspace=workspace, stream=stream, clear_err=True)
    st = lib.gr_beam_step(ctypes.byref(desc), ctypes.byref(io), ctypes.c_void_p(ws.data_ptr()),
                          ctypes.c_size_t(ws.numel()), ctypes.c_void_p(s.cuda_stream))
    _lib.check(st, "gr_beam_step")
    return out


class BeamSearchSampler:
    """Beam-search sampler for catalog-constrained generative recommendation.

    Holds the step configuration, the device copy of the catalog trie and a
    reusable workspace.  ``step`` advances all requests by one token."""

    def __init__(self, beam_width: int, *, vocab_size: int, catalog=None, logprobs_mode: str = "raw_logprobs",
                 per_beam_k: int = 0, eos_token_id: Optional[int] = None, device=None):
        if logprobs_mode not in LOGPROBS_MODES:
            raise ValueError(f"logprobs_mode must be one of {sorted(LOGPROBS_MODES)}")
        self.beam_width = int(beam_width)
        self.vocab_size = int(vocab_size)
        self.logprobs_mode = logprobs_mode
        self.per_beam_k = int(per_beam_k)
        self.eos_token_id = eos_token_id
        self.device = torch.device(device if device is not None else "cuda")
        self.workspace = Workspace(self.device)
        self.csr = None
        if catalog is not None:
            trie = getattr(catalog, "csr", catalog)
            trie.validate(self.vocab_size)
            self.csr = (torch.from_numpy(trie.row_ptr).to(self.device),
                        torch.from_numpy(trie.child_tok).to(self.device),
                        torch.from_numpy(trie.child_node).to(self.device))

    def step(self, logits, cum, node, hist=None, *, vocab_offset: int = 0, temperature=None,
             repetition_penalty=None, presence_penalty=None, frequency_penalty=None, stream=None) -> BeamStepOutput:
        return beam_step(logits, cum, node, beam_width=self.beam_width, csr=self.csr, vocab_size=self.vocab_size,
                         vocab_offset=vocab_offset, logprobs_mode=self.logprobs_mode, per_beam_k=self.per_beam_k,
                         eos_token_id=self.eos_token_id, hist=hist, temperature=temperature,
                         repetition_penalty=repetition_penalty, presence_penalty=presence_penalty,
                         frequency_penalty=frequency_penalty, workspace=self.workspace, stream=stream)
