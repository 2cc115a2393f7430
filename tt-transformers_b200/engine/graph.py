"""Captured decode steps: the CUDA-graph counterpart of the reference's traced decode.

The reference captures the command stream of a decode step once per lane shape, keeps the
step's inputs in persistent device buffers, refreshes those in place and replays
(src/tt_transformers/llm_runtime/trace_compiler.py:314-541; decode.py:684-819). Here a step
in which every request brings exactly one token is padded to the next captured batch size
(padding rows sit at position 0 and write to the scratch page), its metadata is copied into
a persistent device buffer, and the graph captured for that size is replayed. The logits
live in a buffer that the next replay of the same size overwrites.
"""

from __future__ import annotations

import gc
import weakref
from typing import Dict, List

import torch


OWN_ARGMAX = "own argmax"        # token_feedback value: the tokens are the argmax of this graph's replay before


class DecodeGraphs:
    def __init__(self, engine):
        self._engine = weakref.ref(engine)       # no cycle with the engine: both go when the last user lets go
        sizes, b = [], 1
        while b < engine.config.max_batch_size:
            sizes.append(b)
            b *= 2
        sizes.append(engine.config.max_batch_size)
        self.sizes = sizes
        self._graphs: Dict[int, tuple] = {}
        self.replays = 0
        self.pool = None
        self._last_size = None
        self.greedy = None

    @property
    def engine(self):
        return self._engine()

    def _bucket(self, rows: int) -> int:
        for s in self.sizes:
            if s >= rows:
                return s
        raise ValueError(f"{rows} requests exceed the engine's max_batch_size")

    def _capture(self, size: int, entries) -> tuple:
        eng = self.engine
        W = eng.cache.table_width
        host, layout, lists = eng._fill_host(entries, pad_to=size, table_width=W, want_all=True)
        static = torch.empty(layout["total"], dtype=torch.int32, device=eng.runtime.device)
        static.copy_(host, non_blocking=True)
        eng._record_staging()
        lists = dict(lists, max_context=eng.max_seq_len)      # key splits are sized for the longest context
        batch = eng._batch_from(static, layout, lists)
        side = torch.cuda.Stream(device=eng.runtime.device)
        side.wait_stream(torch.cuda.current_stream(eng.runtime.device))
        with torch.cuda.stream(side):                         # warm up outside the capture
            eng.model.forward(batch, eng.cache)
        torch.cuda.current_stream(eng.runtime.device).wait_stream(side)
        torch.cuda.synchronize(eng.runtime.device)
        graph = torch.cuda.CUDAGraph()
        before = eng.kernels.launches
        batch.extras.clear()
        # No garbage collection while the stream is capturing: an object that happens to be collected then
        # (an engine used before, with its pinned buffers, events and graphs) would make CUDA calls that
        # are not allowed during a capture and invalidate it.
        gc_was_on = gc.isenabled()
        gc.disable()                  # (torch.cuda.graph collects once on entry, before the capture begins)
        try:
            with torch.cuda.graph(graph, pool=self.pool):
                logits = eng.model.forward(batch, eng.cache)
                # the greedy choice of every row, left where the next replay's embedding looks for its tokens:
                # a greedy decode loop then needs neither a sampling launch nor a copy between two replays
                greedy = eng.kernels.sample(logits)
                static[layout["o_tok"]:layout["o_tok"] + size].copy_(greedy)
        finally:
            if gc_was_on:
                gc.enable()
        if self.pool is None:
            self.pool = graph.pool()
        kernels_in_graph = eng.kernels.launches - before
        return graph, static, layout, logits, kernels_in_graph, greedy

    def run(self, entries: List, token_feedback: torch.Tensor = None) -> torch.Tensor:
        """Replay the captured step for these entries. With token_feedback (int32 on the device, one
        token per entry, typically what the sampler wrote for the step before) the token ids come
        from there instead of from the entries, so the host need not have seen them yet."""
        eng = self.engine
        rows = len(entries)
        size = self._bucket(rows)
        if size not in self._graphs:
            self._graphs[size] = self._capture(size, entries)
        graph, static, layout, logits, kernels_in_graph, greedy = self._graphs[size]
        host, new_layout, _ = eng._fill_host(entries, pad_to=size, table_width=eng.cache.table_width, want_all=True)
        assert new_layout["total"] == layout["total"]
        if isinstance(token_feedback, str) and token_feedback == OWN_ARGMAX:
            if self._last_size != size:
                raise ValueError("OWN_ARGMAX needs the step before to have been a replay of the same captured size")
            first = layout["o_pos"]                     # everything but the token ids, which the replay before left in place
            static[first:].copy_(host[first:], non_blocking=True)
            eng.h2d_bytes += 4 * (host.numel() - first)
        else:
            static.copy_(host, non_blocking=True)
            eng.h2d_bytes += 4 * host.numel()
        eng._record_staging()
        if torch.is_tensor(token_feedback):
            static[layout["o_tok"]:layout["o_tok"] + rows].copy_(token_feedback[:rows])
        graph.replay()
        self._last_size = size
        self.greedy = greedy[:rows]                     # overwritten by the next replay of this size
        eng.kernels.launches += kernels_in_graph
        self.replays += 1
        want = [i for i, e in enumerate(entries) if len(e.want)]
        if len(want) == rows:
            return logits[:rows]
        return logits[torch.tensor(want, dtype=torch.long, device=logits.device)] if want else logits[:0]
