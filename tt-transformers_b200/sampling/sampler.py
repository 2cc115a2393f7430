"""From the logits of a step to one token per request, on the device.

One call of the sampling kernel serves a batch in which every row has its own
temperature, top_k, top_p, seed and counter. The random number of a row depends only on
(seed, counter), the counter being the index of the token in the request's output, so a
request draws the same tokens wherever it sits in a batch and however its prompt was cut
(the reference's per-request stream: src/tt_transformers/modules/sampling/seed_manager_1d.py:40-55).
"""

from __future__ import annotations

from typing import List, Sequence

import torch

from .params import SamplingParams


class Sampler:
    def __init__(self, kernels, device):
        self.kernels, self.device = kernels, torch.device(device)
        self.max_top_k = int(getattr(kernels, "max_top_k", 64))

    def validate(self, params: SamplingParams) -> None:
        """Every combination of temperature, top_k and top_p is served: up to `max_top_k` candidates are
        selected one by one, more (or top_p alone) by thresholds on the logit's value."""
        if not isinstance(params, SamplingParams):
            raise TypeError(f"sampling parameters must be SamplingParams, got {type(params).__name__}")

    def sample(self, logits: torch.Tensor, params: Sequence[SamplingParams], seeds: Sequence[int],
               counters: Sequence[int]) -> List[int]:
        """logits float32 [rows, vocab]; one token id per row, on the host."""
        if logits.shape[0] == 0:
            return []
        return self.sample_device(logits, params, seeds, counters).tolist()

    def sample_device(self, logits: torch.Tensor, params: Sequence[SamplingParams], seeds: Sequence[int],
                      counters: Sequence[int]) -> torch.Tensor:
        """The same, but the ids stay on the device (int32 [rows]): nothing waits for the GPU."""
        if all(p.greedy for p in params):
            return self.kernels.sample(logits)
        pinned = self.device.type == "cuda"
        f = torch.tensor([[p.temperature for p in params], [p.top_p for p in params]], dtype=torch.float32,
                         pin_memory=pinned).to(self.device, non_blocking=True)
        i = torch.tensor([[p.top_k for p in params], list(counters)], dtype=torch.int32,
                         pin_memory=pinned).to(self.device, non_blocking=True)
        s = torch.tensor([int(x) & 0x7FFFFFFFFFFFFFFF for x in seeds], dtype=torch.int64,
                         pin_memory=pinned).to(self.device, non_blocking=True)
        return self.kernels.sample(logits, f[0], i[0], f[1], s, i[1])
