"""B200-native constrained beam-search step of vLLM-GR (sm_100a CUDA behind a C ABI)."""
__version__ = "0.1.0"
