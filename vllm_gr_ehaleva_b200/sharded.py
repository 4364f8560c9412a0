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
from .sample.beam_search_sampler import BeamStepOutput, Workspace, _prepare

__all__ = ["lse_partials", "shard_candidates", "merge_candidates", "sharded_beam_step", "torch_all_gather"]


def _call(name, fn, *args):
    _lib.check(fn(*args), name)


def lse_partials(local_logits: torch.Tensor, cum: torch.Tensor, node: torch.Tensor, **kw) -> torch.Tensor:
    """Phase 1: float32 [R*NB, 2] = (max, sum exp(y - max)) over the local columns."""
    lib = _lib.load()
    desc, io, out, ws, s, _keep = _prepare(local_logits, cum, node, **kw)
    R, NB = out.lse.shape
    partials = torch.empty((R * NB, 2), dtype=torch.float32, device=local_logits.device)
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
    _call("gr_merge_candidates", lib.gr_merge_candidates, ctypes.byref(desc), ctypes.byref(io),
          ctypes.c_void_p(gathered_keys.data_ptr()), ctypes.c_int32(S), ctypes.c_void_p(ws.data_ptr()),
          ctypes.c_size_t(ws.numel()), ctypes.c_void_p(s.cuda_stream))
    return out


def sharded_beam_step(local_logits: torch.Tensor, cum: torch.Tensor, node: torch.Tensor, *,
                      all_gather: Callable[[torch.Tensor], torch.Tensor], beam_width: int, vocab_size: int,
                      vocab_offset: int, csr=None, eos_token_id: Optional[int] = None,
                      hist: Optional[torch.Tensor] = None, logprobs_mode: str = "raw_logprobs",
                      temperature=None, repetition_penalty=None, presence_penalty=None, frequency_penalty=None,
                      workspace: Optional[Workspace] = None,
                      stream: Optional[torch.cuda.Stream] = None) -> BeamStepOutput:
    """One constrained beam step over vocabulary-sharded logits; every rank
    returns the same outputs.  eos_score comes from the rank whose columns hold
    the EOS token (NaN elsewhere, so the first non-NaN over ranks is taken)."""
    kw = dict(beam_width=beam_width, csr=csr, vocab_size=vocab_size, vocab_offset=vocab_offset,
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
