"""Worker-side pieces of the mega-request decode: the logprobs remux and the
device beam step with device-resident beam state."""
from .beam_hook import WorkerBeamHook, step_runs
from .remux import remux_logprobs_tensors

__all__ = ["WorkerBeamHook", "remux_logprobs_tensors", "step_runs"]
