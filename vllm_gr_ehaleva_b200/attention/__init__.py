"""Attention-side pieces of the beam-consecutive decode (suffix KV gather)."""
from .suffix_kv import extract_suffix_kv, gather_desc

__all__ = ["extract_suffix_kv", "gather_desc"]
