"""Attention-side pieces of the beam-consecutive decode (suffix KV gather)."""
from .suffix_kv import build_suffix_metadata, extract_suffix_kv, gather_desc, suffix_records

__all__ = ["build_suffix_metadata", "extract_suffix_kv", "gather_desc", "suffix_records"]
