"""Per-request sampling parameters.

Names and meanings follow the reference: temperature 0 means greedy, top_k and top_p
restrict the candidates, seed fixes the request's random stream
(src/tt_transformers/sampling/sampling_params.py:9-24; normalisation
src/tt_transformers/modules/sampling/params.py:196-205). Any top_k is taken, and top_p cuts
over the whole vocabulary when top_k is 0, as the reference's host sampler does
(src/tt_transformers/models/hf_generation.py:138-146). Penalties and log-probs, which the
reference's device sampler also has, are not part of this engine.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple


@dataclass(frozen=True)
class SamplingParams:
    temperature: float = 0.0            # 0: greedy (largest logit, lowest id among equals)
    top_k: int = 0                      # 0: all tokens; else the k largest logits
    top_p: float = 1.0                  # < 1: the low tail of cumulative probability 1 - top_p is cut (of the top_k, if given)
    seed: Optional[int] = None          # None: derived from the request's arrival number
    max_new_tokens: int = 128
    eos_token_ids: Tuple[int, ...] = ()
    ignore_eos: bool = False

    def __post_init__(self):
        if self.temperature < 0:
            raise ValueError(f"temperature must not be negative, got {self.temperature}")
        if self.top_k < 0:
            raise ValueError(f"top_k must not be negative, got {self.top_k}")
        if not 0.0 <= self.top_p <= 1.0:
            raise ValueError(f"top_p must lie in [0, 1], got {self.top_p}")
        if self.max_new_tokens < 0:
            raise ValueError("max_new_tokens must not be negative")

    @property
    def greedy(self) -> bool:
        return self.temperature == 0.0
