"""Vocab-sharded beam step (logit columns split over ranks).

With a column-parallel lm_head each rank holds columns
[vocab_offset, vocab_offset + V_l) of every beam's logits row; vLLM would
all-gather the full rows before its sampler (vllm logits_processor.py:75-86).
Here a step is three device calls with two small all-gathers between them:

  1. ``lse_partials``      per-row (max, sum exp) over the local columns
     all-gather            R*NB*8 bytes per rank
  2. ``shard_candidates``  global lse from the gathered partials, this rank's
                           catalog children scored, its canonical top-2B keys
                           per request
     all-gather            R*2B*8 bytes per rank
  3. ``merge_candidates``  the global top-2B per request, new beams, child
                           nodes and the forked token table (same on every rank)

``all_gather(t)`` returns the ranks' tensors stacked in rank order (shard k
first along dim 0); ``torch_all_gather(group)`` builds one from a
torch.distributed process group (NCCL on GPUs).  Tests on one GPU pass a
function that stacks the shards' results directly.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

import torch

from . import _lib
from .sample.beam_search_sampler import BeamStepOutput, Workspace, _launch_stream, _prepare

__all__ = ["lse_partials", "shard_candidates", "merge_candidates", "sharded_beam_step", "torch_all_gather"]


def _call(name, fn, *args):
    _lib.check(fn(*args), name)


def lse_partials(local_logits: torch.Tensor, cum: torch.Tensor, node: torch.Tensor, **kw) -> torch.Tensor:
    """Phase 1: float32 [R*NB, 2] = (max, sum exp(y - max)) over the local columns."""
    lib = _lib.load()
    desc, io, out, ws, s, _keep = _prepare(local_logits, cum, node, **kw)
    R, NB = out.lse.shape
    partials = torch.empty((R * NB, 2), dtype=torch.float32, device=local_logits.device)
    s = _launch_stream(kw.get("stream"), local_logits.device, (partials,))
    _call("gr_lse_partials", lib.gr_lse_partials, ctypes.byref(desc), ctypes.byref(io),
          ctypes.c_void_p(partials.data_ptr()), ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()),
          ctypes.c_void_p(s.cuda_stream))
    partials.err = out.err            # device error word of this call
    return partials


def shard_candidates(local_logits: torch.Tensor, cum: torch.Tensor, node: torch.Tensor,
                     gathered_partials: torch.Tensor, **kw):
    """Phase 2: (keys int64 [R, 2B] zero padded, lse [R, NB], eos_score [R, NB], err)."""
    lib = _lib.load()
    desc, io, out, ws, s, _keep = _prepare(local_logits, cum, node, **kw)
    R = out.lse.shape[0]
    k2 = out.cand_score.shape[1]
    S = int(gathered_partials.shape[0])
    gathered_partials = gathered_partials.to(torch.float32).contiguous()
    keys = torch.empty((R, k2), dtype=torch.int64, device=local_logits.device)
    s = _launch_stream(kw.get("stream"), local_logits.device, (gathered_partials, keys))
    _call("gr_shard_candidates", lib.gr_shard_candidates, ctypes.byref(desc), ctypes.byref(io),
          ctypes.c_void_p(gathered_partials.data_ptr()), ctypes.c_int32(S), ctypes.c_void_p(keys.data_ptr()),
          ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()), ctypes.c_void_p(s.cuda_stream))
    return keys, out.lse, out.eos_score, out.err


def merge_candidates(local_logits: torch.Tensor, cum: torch.Tensor, node: torch.Tensor,
                     gathered_keys: torch.Tensor, **kw) -> BeamStepOutput:
    """Phase 3: the step's outputs from every rank's top-2B keys ([S, R, 2B])."""
    lib = _lib.load()
    desc, io, out, ws, s, _keep = _prepare(local_logits, cum, node, **kw)
    S = int(gathered_keys.shape[0])
    gathered_keys = gathered_keys.to(torch.int64).contiguous()
    s = _launch_stream(kw.get("stream"), local_logits.device, (gathered_keys,))
    _call("gr_merge_candidates", lib.gr_merge_candidates, ctypes.byref(desc), ctypes.byref(io),
          ctypes.c_void_p(gathered_keys.data_ptr()), ctypes.c_int32(S), ctypes.c_void_p(ws.data_ptr()),
          ctypes.c_size_t(ws.numel()), ctypes.c_void_p(s.cuda_stream))
    return out


def sharded_beam_step(local_logits: torch.Tensor, cum: torch.Tensor, node: torch.Tensor, *,
                      all_gather: Callable[[torch.Tensor], torch.Tensor], beam_width: int, vocab_size: int,
                      vocab_offset: int, vocab_stride: int = 1, csr=None, eos_token_id: Optional[int] = None,
                      hist: Optional[torch.Tensor] = None, logprobs_mode: str = "raw_logprobs",
                      temperature=None, repetition_penalty=None, presence_penalty=None, frequency_penalty=None,
                      workspace: Optional[Workspace] = None,
                      stream: Optional[torch.cuda.Stream] = None) -> BeamStepOutput:
    """One constrained beam step over vocabulary-sharded logits; every rank
    returns the same outputs.  Local column j holds token vocab_offset +
    j * vocab_stride (a contiguous slice, or shard k = vocab_offset of a
    strided split over vocab_stride ranks).  eos_score comes from the rank
    whose columns hold the EOS token (NaN elsewhere, so the first non-NaN over
    ranks is taken)."""
    kw = dict(beam_width=beam_width, csr=csr, vocab_size=vocab_size, vocab_offset=vocab_offset,
              vocab_stride=vocab_stride,
              logprobs_mode=logprobs_mode, per_beam_k=0, eos_token_id=eos_token_id, hist=hist,
              temperature=temperature, repetition_penalty=repetition_penalty, presence_penalty=presence_penalty,
              frequency_penalty=frequency_penalty, workspace=workspace, stream=stream)
    partials = lse_partials(local_logits, cum, node, **kw)
    err = partials.err
    gathered_partials = all_gather(partials)
    keys, lse, eos_score, err2 = shard_candidates(local_logits, cum, node, gathered_partials, **kw)
    gathered_keys = all_gather(keys)
    out = merge_candidates(local_logits, cum, node, gathered_keys, **kw)
    out.lse = lse
    if eos_token_id is not None:
        eos_all = all_gather(eos_score)
        eos = eos_all[0]
        for k in range(1, eos_all.shape[0]):
            eos = torch.where(torch.isnan(eos), eos_all[k], eos)
        out.eos_score = eos
    else:
        out.eos_score = eos_score
    out.err = out.err | err | err2
    return out


def torch_all_gather(group=None) -> Callable[[torch.Tensor], torch.Tensor]:
    """all_gather over a torch.distributed group: [S, *shape] in rank order."""
    import torch.distributed as dist

    def gather(t: torch.Tensor) -> torch.Tensor:
        t = t.contiguous()
        world = dist.get_world_size(group)
        if dist.get_backend(group) == "nccl":
            out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(out, t, group=group)
            return out
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t, group=group)
        return torch.stack(parts)
    return gather


class ShardedStepper:
    """The vocab-sharded step for one batch shape, with its descriptor, device
    buffers and gather targets built once, so that a step costs three library
    calls and two all-gathers on the host.  Outputs alternate between two
    buffer sets: a step's outputs stay valid while the next step runs (they can
    be its inputs) and are overwritten by the step after that."""

    def __init__(self, *, num_requests: int, num_beams: int, beam_width: int, vocab_size: int, vocab_local: int,
                 vocab_offset: int, num_shards: int, csr, hist_len: int, vocab_stride: int = 1,
                 logits_dtype=torch.bfloat16,
                 row_stride: Optional[int] = None, eos_token_id: Optional[int] = None,
                 all_gather: Optional[Callable[[torch.Tensor], torch.Tensor]] = None, group=None, device=None):
        from .sample.beam_search_sampler import _DTYPES, make_desc, workspace_size
        self.lib = _lib.load()
        self.device = torch.device(device if device is not None else "cuda")
        R, NB, B, S = int(num_requests), int(num_beams), int(beam_width), int(num_shards)
        self.R, self.NB, self.B, self.S, self.T = R, NB, B, S, int(hist_len)
        row_ptr, child_tok, child_node = csr
        self.csr = csr
        self.eos = eos_token_id
        self.desc = make_desc(R=R, NB=NB, B=B, V=int(vocab_size), VL=int(vocab_local), voff=int(vocab_offset),
                              row_stride=int(row_stride if row_stride is not None else vocab_local),
                              dtype=_DTYPES[logits_dtype], mode=_lib.LOGPROBS_RAW, K=0,
                              eos=-1 if eos_token_id is None else int(eos_token_id), T=self.T,
                              N=int(row_ptr.numel()) - 1, E=int(child_tok.numel()), VS=int(vocab_stride))
        dev = dict(device=self.device)
        f32, i32 = dict(dtype=torch.float32, **dev), dict(dtype=torch.int32, **dev)
        self.outs = [BeamStepOutput(
            cand_score=torch.empty((R, 2 * B), **f32), cand_token=torch.empty((R, 2 * B), **i32),
            cand_parent=torch.empty((R, 2 * B), **i32), sel_score=torch.empty((R, B), **f32),
            sel_token=torch.empty((R, B), **i32), sel_parent=torch.empty((R, B), **i32),
            sel_node=torch.empty((R, B), **i32), eos_score=torch.empty((R, NB), **f32),
            hist_out=torch.empty((R, B, self.T + 1), **i32), lse=torch.empty((R, NB), **f32),
            err=torch.zeros(1, **i32)) for _ in range(2)]
        self.partials = torch.empty((R * NB, 2), **f32)
        self.keys = torch.empty((R, 2 * B), dtype=torch.int64, **dev)
        self.gathered_p = torch.empty((S, R * NB, 2), **f32)
        self.gathered_k = torch.empty((S, R, 2 * B), dtype=torch.int64, **dev)
        self.eos_all = torch.empty((S, R, NB), **f32)
        self.ws = torch.empty(max(workspace_size(self.desc), 256), dtype=torch.uint8, **dev)
        self.group = group
        self.gather_fn = all_gather
        self.k = 0

    def _gather(self, dst: torch.Tensor, src: torch.Tensor) -> None:
        if self.gather_fn is not None:
            dst.copy_(self.gather_fn(src))
            return
        import torch.distributed as dist
        dist.all_gather_into_tensor(dst, src, group=self.group)

    def step(self, local_logits: torch.Tensor, cum: torch.Tensor, node: torch.Tensor,
             hist: Optional[torch.Tensor] = None, marks: Optional[list] = None) -> BeamStepOutput:
        """One step.  `marks`: six CUDA events to record on the current stream
        around the phases (start, lse partials, their all-gather, shard
        candidates, their all-gather, merge), for timing them apart."""
        def mark(i):
            if marks is not None:
                marks[i].record()
        out = self.outs[self.k & 1]
        self.k += 1
        io = _lib.StepIO()
        row_ptr, child_tok, child_node = self.csr
        vp = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731
        io.logits, io.cum, io.node, io.hist_in = vp(local_logits), vp(cum), vp(node), vp(hist)
        io.row_ptr, io.child_tok, io.child_node = vp(row_ptr), vp(child_tok), vp(child_node)
        io.cand_score, io.cand_token, io.cand_parent = vp(out.cand_score), vp(out.cand_token), vp(out.cand_parent)
        io.sel_score, io.sel_token, io.sel_parent, io.sel_node = (vp(out.sel_score), vp(out.sel_token),
                                                                   vp(out.sel_parent), vp(out.sel_node))
        io.eos_score, io.hist_out, io.lse, io.err = vp(out.eos_score), vp(out.hist_out), vp(out.lse), vp(out.err)
        out.err.zero_()
        s = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        d, iop = ctypes.byref(self.desc), ctypes.byref(io)
        wsp, wsn = ctypes.c_void_p(self.ws.data_ptr()), ctypes.c_size_t(self.ws.numel())
        mark(0)
        _lib.check(self.lib.gr_lse_partials(d, iop, vp(self.partials), wsp, wsn, s), "gr_lse_partials")
        mark(1)
        self._gather(self.gathered_p, self.partials)
        mark(2)
        _lib.check(self.lib.gr_shard_candidates(d, iop, vp(self.gathered_p), ctypes.c_int32(self.S), vp(self.keys),
                                                wsp, wsn, s), "gr_shard_candidates")
        mark(3)
        self._gather(self.gathered_k, self.keys)
        mark(4)
        _lib.check(self.lib.gr_merge_candidates(d, iop, vp(self.gathered_k), ctypes.c_int32(self.S), wsp, wsn, s),
                   "gr_merge_candidates")
        mark(5)
        if self.eos is not None:
            self._gather(self.eos_all, out.eos_score)
            eos = self.eos_all[0]
            for k in range(1, self.S):
                eos = torch.where(torch.isnan(eos), self.eos_all[k], eos)
            out.eos_score.copy_(eos)
        return out
