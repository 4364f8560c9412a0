"""Mega-request step update with the fork table as int32 arrays.

Every decode step of a mega request, the reference sends the engine core one
MegaRequestStepUpdate (vllm_gr/v1/engine/types.py:48-71), built in Python by
serving_engine.py:91-168: per new beam a parent id string, a child id string
and the beam's full token list since the prompt, plus the ids of the previous
beams that no child forked from.  Every beam id follows one rule,
f"{batch}-beam-{index}" (serving_engine.py:72, 115), so the same content fits
in two batch ids, the parents' indices and one int32 token table — which is
what the device step already produces (sel_parent and the fork table
hist_out), copied to the host in one piece.

`MegaStepFork` is that message.  `step_update_fields` gives back the
reference message's fields (for a consumer written against it) and
`mega_token_ids` the token list the core builds from it
(vllm_gr/v1/engine/core.py:109-112).  The request's SamplingParams do not
change across its steps: they travel as msgpack bytes encoded once by the
caller (`encode_params`) instead of being re-encoded every step.
"""
from __future__ import annotations

from collections.abc import Mapping

import msgspec
import numpy as np


class MegaStepFork(msgspec.Struct, array_like=True, omit_defaults=True, gc=False):
    """One decode step of a mega request.  parents[i] (int32) is the index,
    among the previous step's beams, of new beam i's parent; tokens is the
    int32 [beam_width, steps] table of each new beam's tokens after the prompt
    prefix.  Beam ids are f"{batch_id}-beam-{i}" (new beams) and
    f"{prev_batch_id}-beam-{j}" (previous beams, j < prev_width)."""
    session_id: str
    batch_id: str
    prev_batch_id: str
    prev_width: int
    beam_width: int
    prefix_len: int
    steps: int
    parents: bytes
    tokens: bytes
    sampling_params: bytes = b""
    eos_token_id: int | None = None
    client_index: int = 0
    current_wave: int = 0
    priority: int = 0
    data_parallel_rank: int | None = None
    cache_salt: str | None = None
    trace_headers: Mapping[str, str] | None = None


_ENC = msgspec.msgpack.Encoder()
_DEC = msgspec.msgpack.Decoder(MegaStepFork)


def encode_params(sampling_params) -> bytes:
    """A SamplingParams (vLLM's msgspec struct) as msgpack bytes, once per request."""
    return msgspec.msgpack.encode(sampling_params)


def decode_params(raw: bytes):
    from vllm.sampling_params import SamplingParams
    return msgspec.msgpack.decode(raw, type=SamplingParams)


def build_step_fork(session_id: str, batch_id: str, prev_batch_id: str, prev_width: int, parents, tokens,
                    prefix_len: int, **fields) -> MegaStepFork:
    """parents: int [W] (one request's sel_parent); tokens: int [W, steps] (its beams'
    tokens after the prefix, e.g. the fork table hist_out).  Host arrays or
    anything numpy can read; other MegaStepFork fields by keyword."""
    p = np.ascontiguousarray(np.asarray(parents), dtype="<i4")
    t = np.ascontiguousarray(np.asarray(tokens), dtype="<i4")
    if p.ndim != 1 or t.ndim != 2 or t.shape[0] != p.shape[0]:
        raise ValueError(f"parents [W] and tokens [W, steps] expected, got {p.shape} and {t.shape}")
    if p.size and (p.min() < 0 or p.max() >= prev_width):
        raise ValueError(f"parent index outside [0, {prev_width})")
    return MegaStepFork(session_id=session_id, batch_id=batch_id, prev_batch_id=prev_batch_id,
                        prev_width=int(prev_width), beam_width=int(p.shape[0]), prefix_len=int(prefix_len),
                        steps=int(t.shape[1]), parents=p.tobytes(), tokens=t.tobytes(), **fields)


def encode(fork: MegaStepFork) -> bytes:
    return _ENC.encode(fork)


def decode(raw: bytes) -> MegaStepFork:
    return _DEC.decode(raw)


def parents_of(fork: MegaStepFork) -> np.ndarray:
    return np.frombuffer(fork.parents, dtype="<i4")


def tokens_of(fork: MegaStepFork) -> np.ndarray:
    return np.frombuffer(fork.tokens, dtype="<i4").reshape(fork.beam_width, fork.steps)


def step_update_fields(fork: MegaStepFork) -> dict:
    """The reference MegaRequestStepUpdate's content (serving_engine.py:108-142):
    parent and child beam ids, per-beam token lists, pruned parent ids."""
    parents = parents_of(fork)
    prev = [f"{fork.prev_batch_id}-beam-{j}" for j in range(fork.prev_width)]
    used = np.zeros(fork.prev_width, bool)
    used[parents] = True
    return dict(session_id=fork.session_id,
                parent_beam_ids=[prev[j] for j in parents.tolist()],
                child_beam_ids=[f"{fork.batch_id}-beam-{i}" for i in range(fork.beam_width)],
                beam_tokens=tokens_of(fork).tolist(),
                pruned_ids=[prev[j] for j in range(fork.prev_width) if not used[j]],
                prefix_len=fork.prefix_len, beam_width=fork.beam_width, eos_token_id=fork.eos_token_id)


def mega_token_ids(fork: MegaStepFork, prefill_tokens) -> np.ndarray:
    """The mega request's prompt as the engine core builds it
    (vllm_gr/v1/engine/core.py:109-112): the shared prefill, then every beam's
    tokens in beam order."""
    return np.concatenate([np.asarray(prefill_tokens, dtype=np.int64), tokens_of(fork).astype(np.int64).ravel()])
