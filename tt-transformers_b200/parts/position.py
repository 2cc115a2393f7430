"""Position encodings.

`rotary`: rotation frequencies theta^(-2i/d), optionally with Llama-3 per-frequency
scaling (src/tt_transformers/models/llama3_8b/hf_generator.py:88-120). The frequencies
are computed once, in float32, by the same sequence of float32 operations that the
reference uses; the angles position x frequency and their sines and cosines are
computed in the kernels, in float32, from the positions of each step.
`none`: nothing is rotated (for mixers that carry order by themselves).
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from .base import PositionEncoding, register_part


def rotary_inverse_frequencies(rotary_dim: int, theta: float, scaling: Optional[dict]) -> torch.Tensor:
    exponents = torch.arange(0, rotary_dim, 2, dtype=torch.float32) / rotary_dim
    inv_freq = 1.0 / (theta ** exponents)
    if scaling is None:
        return inv_freq
    factor = float(scaling["factor"])
    low, high = float(scaling["low_freq_factor"]), float(scaling["high_freq_factor"])
    original = float(scaling["original_max_position_embeddings"])
    scaled = []
    for freq in inv_freq:                      # element by element, as float32 scalars
        wavelength = 2 * math.pi / freq
        if wavelength < original / high:       # short waves keep their frequency
            scaled.append(freq)
        elif wavelength > original / low:      # long waves are slowed down by the factor
            scaled.append(freq / factor)
        else:                                  # between the two: a linear blend
            blend = (original / wavelength - low) / (high - low)
            scaled.append((1 - blend) * freq / factor + blend * freq)
    return torch.stack([torch.as_tensor(s, dtype=torch.float32) for s in scaled])


class Rotary(PositionEncoding):
    """`interleaved` False pairs element i of a head with element i + rotary_dim/2 (the row order of the
    checkpoints this engine reads); True pairs 2i with 2i + 1, the order on which the reference rotates after
    permuting the checkpoint's rows (src/tt_transformers/models/llama32_1b/weight_utils.py:23-25)."""

    def __init__(self, rotary_dim: int, theta: float, scaling: Optional[dict] = None, interleaved: bool = False):
        if rotary_dim % 2:
            raise ValueError(f"rotary_dim must be even, got {rotary_dim}")
        self.rotary_dim, self.theta, self.scaling = int(rotary_dim), float(theta), scaling
        self.interleaved = bool(interleaved)
        self.inv_freq_host = rotary_inverse_frequencies(self.rotary_dim, self.theta, scaling)

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.inv_freq = self.inv_freq_host.to(runtime.device)

    def rotation(self):
        return self.inv_freq, self.rotary_dim


class NoPosition(PositionEncoding):
    def __init__(self):
        pass


register_part("position", "rotary", Rotary)
register_part("position", "none", NoPosition)
