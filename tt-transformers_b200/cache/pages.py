"""A pool of page numbers with a free list.

Page 0 is never handed out: block-table entries that cover nothing point at it, and
padded rows of a captured decode step write there. The lowest-numbered free page is handed
out first: a freed page is used again at once (a small pool shows stale contents in tests),
and a request's pages tend to ascend in memory, which the attention kernels read measurably
faster than a descending or scattered order. The reference has no allocator of its own: it
hands out contiguous ranges per call (src/tt_transformers/models/hf_generation.py:337-348).
"""

from __future__ import annotations

import heapq
from typing import List, Optional


class PagePoolError(RuntimeError):
    """A page was freed twice or never belonged to the pool."""


class PagePool:
    def __init__(self, num_pages: int):
        if num_pages < 1:
            raise ValueError("a pool needs at least one page")
        self.num_pages = num_pages                    # usable pages are 1 .. num_pages
        self._free: List[int] = list(range(1, num_pages + 1))     # a heap: the smallest number comes first
        self._held = [False] * (num_pages + 1)

    @property
    def free_count(self) -> int:
        return len(self._free)

    @property
    def held_count(self) -> int:
        return self.num_pages - len(self._free)

    def allocate(self, count: int) -> Optional[List[int]]:
        """`count` pages, or None (and nothing taken) if fewer are free."""
        if count < 0:
            raise ValueError("count must not be negative")
        if count > len(self._free):
            return None
        pages = [heapq.heappop(self._free) for _ in range(count)]
        for p in pages:
            self._held[p] = True
        return pages

    def free(self, pages) -> None:
        for p in pages:
            if not 1 <= p <= self.num_pages or not self._held[p]:
                raise PagePoolError(f"page {p} is not held and cannot be freed")
            self._held[p] = False
            heapq.heappush(self._free, p)
