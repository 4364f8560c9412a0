"""Beam-search sampler for catalog-constrained generative recommendation (device step)."""
from .beam_search_sampler import BeamSearchSampler, BeamStepOutput, beam_step, workspace_size  # noqa: F401
