"""The engine's own settings: precision, cache geometry, batch limits.

The counterparts in the reference are its frozen runtime dataclasses
(src/tt_transformers/llm_runtime/config.py:18-159: TraceConfig, PagedKVCacheConfig)
and the loader's arguments max_batch_size / max_seq_len
(src/tt_transformers/models/llama32_1b/hf_generator.py:380-394).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

from .base import ConfigError


@dataclass(frozen=True)
class EngineConfig:
    dtype: str = "bfloat16"              # "bfloat16" (serving) or "float32" (true 32-bit everywhere)
    page_size: int = 16                  # tokens per cache page
    num_pages: Optional[int] = None      # pages per cache group; None: from gpu_memory_fraction, else max_batch_size * max_seq_len
    gpu_memory_fraction: Optional[float] = None   # with num_pages None: the cache may fill the device up to this share of its memory
    max_batch_size: int = 32             # most requests live at a time (slots)
    max_seq_len: int = 4096              # most tokens one request may hold
    max_step_tokens: int = 2048          # token budget of one step
    max_chunk_tokens: int = 2048         # largest prompt portion in one step
    cuda_graph: bool = True              # replay pure-decode steps (and short lone prompts) from captured graphs
    graph_batch_sizes: Optional[Tuple[int, ...]] = None   # batch sizes decode steps are captured at; None: powers of two
    admission: str = "eager"             # "eager": a request starts when its first portion fits; "conservative": when
                                         # prompt + max_new_tokens fit, all reserved at once (it never gives way)
    device: str = "cuda:0"

    def __post_init__(self):
        if self.dtype not in ("bfloat16", "float32"):
            raise ConfigError(f"dtype must be 'bfloat16' or 'float32', got {self.dtype!r}")
        for key in ("page_size", "max_batch_size", "max_seq_len", "max_step_tokens", "max_chunk_tokens"):
            if not isinstance(getattr(self, key), int) or getattr(self, key) < 1:
                raise ConfigError(f"{key} must be a positive integer, got {getattr(self, key)!r}")
        if self.num_pages is not None and self.num_pages < 1:
            raise ConfigError(f"num_pages must be positive, got {self.num_pages}")
        if self.gpu_memory_fraction is not None and not 0.0 < self.gpu_memory_fraction <= 1.0:
            raise ConfigError(f"gpu_memory_fraction must lie in (0, 1], got {self.gpu_memory_fraction}")
        if self.admission not in ("eager", "conservative"):
            raise ConfigError(f"admission must be 'eager' or 'conservative', got {self.admission!r}")
        if self.graph_batch_sizes is not None:
            sizes = tuple(self.graph_batch_sizes)
            if not sizes or any(not isinstance(b, int) or b < 1 for b in sizes) or list(sizes) != sorted(set(sizes)):
                raise ConfigError(f"graph_batch_sizes must be increasing positive integers, got {self.graph_batch_sizes!r}")
            object.__setattr__(self, "graph_batch_sizes", sizes)

    @property
    def pages_per_request(self) -> int:
        return -(-self.max_seq_len // self.page_size)

    def resolved_num_pages(self) -> int:
        if self.num_pages is not None:
            return self.num_pages
        return self.pages_per_request * self.max_batch_size
