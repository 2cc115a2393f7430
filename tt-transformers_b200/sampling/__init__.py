"""Sampling parameters and the sampler that sits on the sampling kernel."""

from .params import SamplingParams
from .sampler import Sampler

__all__ = ["SamplingParams", "Sampler"]
