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

from typing import Optional

import torch

from ..sample.beam_search_sampler import Workspace, beam_step


class SessionState:
    """A session's beams.  After a step the state points into that step's
    batched outputs (row `idx` of the run's tensors), so that a run of the same
    sessions in the same order feeds the next step without copies."""
    __slots__ = ("beam_width", "_own", "_batch", "_idx")

    def __init__(self, beam_width, cum, node, hist):
        self.beam_width = beam_width
        self._own = (cum, node, hist)
        self._batch = None
        self._idx = 0

    @property
    def cum(self):      # float32 [B]
        return self._own[0] if self._batch is None else self._batch["cum"][self._idx]

    @property
    def node(self):     # int32 [B]
        return self._own[1] if self._batch is None else self._batch["node"][self._idx]

    @property
    def hist(self):     # int32 [B, T]: tokens since the prompt (the fork table)
        return self._own[2] if self._batch is None else self._batch["hist"][self._idx]

    def hist_len(self) -> int:
        return self._own[2].shape[1] if self._batch is None else self._batch["hist"].shape[2]


class SessionStep:
    """One session's new beams: row `i` of its run's step outputs (read lazily)."""
    __slots__ = ("_res", "_i")

    def __init__(self, res, i):
        self._res, self._i = res, i

    sel_parent = property(lambda self: self._res.sel_parent[self._i])   # int32 [B]
    sel_token = property(lambda self: self._res.sel_token[self._i])     # int32 [B]
    sel_score = property(lambda self: self._res.sel_score[self._i])     # float32 [B]
    sel_node = property(lambda self: self._res.sel_node[self._i])       # int32 [B]
    hist = property(lambda self: self._res.hist_out[self._i])           # int32 [B, T+1]
    eos_score = property(lambda self: self._res.eos_score[self._i])     # float32 [B] per parent (NaN: none)


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
            T = states[0].hist_len()
            if any(s.hist_len() != T for s in states):
                groups = [([r], first + i * B) for i, r in enumerate(ids)]   # unequal token tables
            else:
                groups = [(ids, first)]
            for gids, row0 in groups:
                st = [self.sessions[r] for r in gids]
                batch = st[0]._batch
                if batch is not None and batch["ids"] == tuple(gids) and all(s._batch is batch for s in st):
                    cum, node, hist = batch["cum"], batch["node"], batch["hist"]   # last step's outputs as they are
                else:
                    cum = torch.stack([s.cum for s in st])
                    node = torch.stack([s.node for s in st])
                    hist = torch.stack([s.hist for s in st]) if T else None
                res = beam_step(logits[row0:row0 + len(gids) * B], cum, node, beam_width=B, csr=self.csr,
                                vocab_size=self.vocab_size, logprobs_mode=self.logprobs_mode,
                                eos_token_id=self.eos_token_id, hist=hist if T else None,
                                workspace=self.workspace)
                new = {"ids": tuple(gids), "cum": res.sel_score, "node": res.sel_node, "hist": res.hist_out}
                for i, r in enumerate(gids):
                    s = self.sessions[r]
                    s._batch, s._idx = new, i
                    out[r] = SessionStep(res, i)
        return out
