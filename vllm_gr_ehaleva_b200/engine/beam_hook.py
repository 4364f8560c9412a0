"""Device beam step inside the worker, with the beam state kept on the device.

In the reference, the worker's sampler returns B*(K+1) logprobs per mega
request (vllm_gr/v1/engine/engine_core_patch.py:527-697, with the remux at
383-445); the serving layer then masks, adds, selects and forks in Python
(serving_engine.py:457-597) and sends the new beams back
(serving_engine.py:91-168).  `WorkerBeamHook` is the worker-side alternative:
it keeps every mega session's beam state (cumulative scores, trie nodes, token
table) on the device, runs the constrained step on the session's logit rows
right where the worker has them, carries the step's outputs (sel_score,
sel_node, hist_out) into the state for the next step, and hands back only the
new beams: parent indices, tokens, scores and the EOS completions — the
content of the int32 step message in vllm_gr_ehaleva_b200.wire.

Logit rows arrive as the worker lays them out: one block of W_logits rows per
request, in `request_row_configs` order (req_id, input_row, W_logits), plain
requests and chunked prefills (W_logits 0 or 1) in between.  Consecutive
mega sessions with the same beam width and a full block of rows form one run
and take one step call on a view of their rows (no copy of the logits).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from ..sample.beam_search_sampler import Workspace, beam_step


@dataclass
class SessionState:
    beam_width: int
    cum: torch.Tensor     # float32 [B]
    node: torch.Tensor    # int32 [B]
    hist: torch.Tensor    # int32 [B, T] tokens since the prompt (the fork table)


@dataclass
class SessionStep:
    sel_parent: torch.Tensor   # int32 [B]
    sel_token: torch.Tensor    # int32 [B]
    sel_score: torch.Tensor    # float32 [B]
    sel_node: torch.Tensor     # int32 [B]
    hist: torch.Tensor         # int32 [B, T+1]
    eos_score: torch.Tensor    # float32 [B] per parent beam (NaN: no EOS candidate)


def step_runs(request_row_configs, sessions) -> list:
    """Group the rows into step calls: [(first row, [req_id, ...], beam_width)] for
    maximal runs of consecutive configs that are registered sessions with a full
    block of beam_width rows and the same beam width, their rows contiguous.
    Other configs (plain requests, partial blocks) are skipped and end a run;
    configs without rows (chunked prefills) do not."""
    runs = []
    row = 0
    cur = None
    for req_id, _input_row, w in request_row_configs:
        s = sessions.get(req_id)
        if s is not None and w == s.beam_width and w > 0:
            if cur is not None and cur[2] == w and cur[0] + len(cur[1]) * w == row:
                cur[1].append(req_id)
            else:
                cur = [row, [req_id], w]
                runs.append(cur)
        elif w > 0:
            cur = None        # rows of another kind in between: the next session starts a new run
        row += w
    return [tuple(r) for r in runs]


class WorkerBeamHook:
    """Per-worker beam state and step.  `csr` is the catalog trie on the device
    (row_ptr, child_tok, child_node); the other arguments are the step's."""

    def __init__(self, *, vocab_size: int, csr=None, eos_token_id: Optional[int] = None,
                 logprobs_mode: str = "raw_logprobs", device=None):
        self.vocab_size = int(vocab_size)
        self.csr = csr
        self.eos_token_id = eos_token_id
        self.logprobs_mode = logprobs_mode
        self.device = torch.device(device if device is not None else "cuda")
        self.workspace = Workspace(self.device)
        self.sessions: dict[str, SessionState] = {}

    def start(self, req_id: str, beam_width: int, cum, node, hist=None) -> None:
        """Register a mega session: its beams' cumulative scores [B], trie nodes [B]
        and tokens since the prompt [B, T] (T may be 0)."""
        B = int(beam_width)
        cum = torch.as_tensor(cum, dtype=torch.float32, device=self.device).reshape(B)
        node = torch.as_tensor(node, dtype=torch.int32, device=self.device).reshape(B)
        hist = (torch.zeros((B, 0), dtype=torch.int32, device=self.device) if hist is None
                else torch.as_tensor(hist, dtype=torch.int32, device=self.device).reshape(B, -1))
        self.sessions[req_id] = SessionState(B, cum, node, hist)

    def end(self, req_id: str) -> None:
        self.sessions.pop(req_id, None)

    def step(self, logits: torch.Tensor, request_row_configs) -> dict:
        """Advance every registered session whose block of rows is in `logits`
        ([rows, V] in the worker's row order).  Returns {req_id: SessionStep};
        the sessions' states now hold the new beams."""
        out = {}
        for first, ids, B in step_runs(request_row_configs, self.sessions):
            states = [self.sessions[r] for r in ids]
            T = states[0].hist.shape[1]
            if any(s.hist.shape[1] != T for s in states):
                # token tables of different lengths: one call per session
                groups = [([r], first + i * B) for i, r in enumerate(ids)]
            else:
                groups = [(ids, first)]
            for gids, row0 in groups:
                st = [self.sessions[r] for r in gids]
                n = len(gids)
                res = beam_step(logits[row0:row0 + n * B], torch.stack([s.cum for s in st]),
                                torch.stack([s.node for s in st]), beam_width=B, csr=self.csr,
                                vocab_size=self.vocab_size, logprobs_mode=self.logprobs_mode,
                                eos_token_id=self.eos_token_id,
                                hist=torch.stack([s.hist for s in st]) if T else None,
                                workspace=self.workspace)
                for i, r in enumerate(gids):
                    s = self.sessions[r]
                    s.cum, s.node, s.hist = res.sel_score[i], res.sel_node[i], res.hist_out[i]
                    out[r] = SessionStep(res.sel_parent[i], res.sel_token[i], res.sel_score[i], res.sel_node[i],
                                         res.hist_out[i], res.eos_score[i])
        return out
