"""Worker-side pieces of the mega-request decode (logprobs remux)."""
from .remux import remux_logprobs_tensors

__all__ = ["remux_logprobs_tensors"]
