"""Beam-search loop driven by the device step (host side).

Mirrors the reference's two loops around its per-step selection:
  online  ``OpenAIServing.beam_search`` (vllm_gr/entrypoints/openai/serving_engine.py:213-645):
          one request, catalog constraint, ``<|sid_begin|>`` appended to the prompt,
          ``<|sid_end|>`` appended to the surviving beams, result tokens without the
          prompt, final sort by cumulative log-prob;
  offline ``LLM.beam_search`` (vllm_gr/entrypoints/llm.py:26-300): several prompts, no
          catalog, result tokens with the prompt, EOS completions keep the EOS token,
          final sort by vLLM's length-penalised score.
Per step the selection (mask, cum add, EOS -> completed, top-B, fork) is one
call of ``step_fn`` over all requests; by default that is the CUDA step
(``sample.beam_step``), which is the product path.

``logits_fn(list_of_token_lists) -> float32 [n, V]`` stands in for the model:
it returns one logits row per beam (in the reference the engine runs the
model on ``beam.tokens``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Optional, Sequence

import numpy as np

from .catalog import NODE_DEAD, NODE_UNCONSTRAINED, CSRTrie


@dataclass
class Beam:
    tokens: list
    cum_logprob: float
    node: int = NODE_UNCONSTRAINED
    finish_reason: Optional[str] = None
    stop_reason: Optional[int] = None


@dataclass
class _Instance:
    prompt_len: int
    beams: list
    completed: list = field(default_factory=list)


def device_step_fn(device="cuda", csr: Optional[CSRTrie] = None, dtype="f32", per_beam_k: int = 0,
                   logprobs_mode: str = "raw_logprobs", temperature: Optional[float] = None):
    """step_fn running the CUDA step; logits are copied to the device per call.
    per_beam_k = beam width gives llm.py's per-beam top-K candidate lists;
    logprobs_mode / temperature are vLLM's (the temperature of the requests'
    SamplingParams, used by the processed mode)."""
    import torch

    from .sample import beam_step
    csr_dev = None
    if csr is not None:
        csr_dev = tuple(torch.from_numpy(a).to(device) for a in (csr.row_ptr, csr.child_tok, csr.child_node))
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dtype]

    def step(logits32, cum, node, *, beam_width, vocab_size, eos_token_id):
        x = torch.from_numpy(np.ascontiguousarray(logits32)).to(device).to(tdt)
        out = beam_step(x, torch.from_numpy(cum).to(device), torch.from_numpy(node).to(device),
                        beam_width=beam_width, csr=csr_dev, vocab_size=vocab_size, per_beam_k=per_beam_k,
                        eos_token_id=None if eos_token_id is None or eos_token_id < 0 else eos_token_id,
                        logprobs_mode=logprobs_mode,
                        temperature=None if temperature is None else [temperature] * cum.shape[0])
        out.check()
        return {k: getattr(out, k).cpu().numpy() for k in ("sel_token", "sel_parent", "sel_score", "sel_node",
                                                          "eos_score")}
    return step


def beam_search(prompts: Sequence[Sequence[int]], logits_fn: Callable, *, beam_width: int, max_tokens: int,
                vocab_size: int, step_fn: Callable, catalog: Optional[CSRTrie] = None,
                begin_token: Optional[int] = None, end_token: Optional[int] = None,
                eos_token_id: Optional[int] = None, ignore_eos: bool = False, online: bool = True,
                length_penalty: float = 1.0, include_stop_str_in_output: bool = False):
    """Returns, per prompt, the best ``beam_width`` finished sequences as
    (tokens, cum_logprob, finish_reason) tuples."""
    B = int(beam_width)
    eos = -1 if (eos_token_id is None or ignore_eos) else int(eos_token_id)
    pre_calc = (1 if begin_token is not None else 0) + (1 if end_token is not None else 0)
    steps = max_tokens - pre_calc
    if steps < 0:
        raise ValueError("max tokens should be not lower than the reserved begin/end tokens")
    insts = []
    for p in prompts:
        toks = list(p) + ([begin_token] if begin_token is not None else [])
        node = NODE_UNCONSTRAINED
        if catalog is not None:
            node = catalog.walk(toks[len(p):])
        insts.append(_Instance(prompt_len=len(p), beams=[Beam(tokens=toks, cum_logprob=0.0, node=node)]))
    for _ in range(steps):
        R = len(insts)
        NB = max(len(i.beams) for i in insts)
        if NB == 0:
            break
        rows = [b.tokens for i in insts for b in i.beams]
        x = np.asarray(logits_fn(rows), dtype=np.float32)
        logits = np.zeros((R, NB, vocab_size), np.float32)
        cum = np.full((R, NB), -np.inf, np.float32)
        node = np.full((R, NB), NODE_DEAD, np.int32)   # padding rows offer no candidates
        k = 0
        for r, inst in enumerate(insts):
            for b, beam in enumerate(inst.beams):
                logits[r, b] = x[k]
                cum[r, b] = beam.cum_logprob
                node[r, b] = beam.node
                k += 1
        out = step_fn(logits, cum, node, beam_width=B, vocab_size=vocab_size, eos_token_id=eos)
        for r, inst in enumerate(insts):
            old = inst.beams
            if eos >= 0:
                for b, beam in enumerate(old):
                    es = float(out["eos_score"][r, b])
                    if not np.isnan(es):      # the beam offered EOS (serving_engine.py:541-562)
                        keep_eos = (not online) or include_stop_str_in_output
                        inst.completed.append(Beam(tokens=beam.tokens + ([eos] if keep_eos else []),
                                                   cum_logprob=es, finish_reason="stop", stop_reason=eos))
            new = []
            for i in range(B):
                p = int(out["sel_parent"][r, i])
                if p < 0:
                    continue
                t = int(out["sel_token"][r, i])
                new.append(Beam(tokens=old[p].tokens + [t], cum_logprob=float(out["sel_score"][r, i]),
                                node=int(out["sel_node"][r, i])))
            inst.beams = new
    results = []
    for inst in insts:
        if end_token is not None:
            for beam in inst.beams:
                beam.tokens.append(end_token)
        done = inst.completed + inst.beams
        if online:
            done = sorted(done, key=lambda s: s.cum_logprob, reverse=True)[:B]
            results.append([(s.tokens[inst.prompt_len:], s.cum_logprob, s.finish_reason or "length") for s in done])
        else:
            def key(s):
                n = len(s.tokens) - (1 if s.tokens and s.tokens[-1] == eos_token_id else 0)
                return s.cum_logprob / (n ** length_penalty)
            done = sorted(done, key=key, reverse=True)[:B]
            results.append([(s.tokens, s.cum_logprob, s.finish_reason) for s in done])
    return results
