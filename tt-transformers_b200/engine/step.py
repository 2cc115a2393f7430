"""The step function: one batch of (request, its next tokens) through the model.

A step takes, for each request in it, the request's next tokens (a portion of its prompt,
cut anywhere, or one decoded token) and the places among them whose logits are wanted.
All entries run as one flat batch: the tokens' keys and values are written into the cache
pages, every token attends to what its request holds in the cache, and float32 logits come
back for the wanted places, in the order of the entries and of `want`. Nothing else is
kept between steps.

The reference has two entry points instead, a padded prefill wave or chunk and a
full-lane decode step, and never mixes them (src/tt_transformers/llm_runtime/execution.py:121-222;
src/tt_transformers/llm_runtime/prefill/plan.py:22-100; src/tt_transformers/llm_runtime/decode.py:1040-1060).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from ..cache import CacheManager, OutOfPages
from ..config.base import read_config_json
from ..config.engine import EngineConfig
from ..parts import DecoderModel, Runtime, StepBatch
from ..registry import architecture_of, get_architecture
from ..weights.loader import check_tensors, read_safetensors

_DTYPES = {"bfloat16": torch.bfloat16, "float32": torch.float32}


@dataclass
class StepEntry:
    request_id: object
    tokens: Sequence[int]
    want: Sequence[int] = field(default_factory=list)     # offsets into `tokens`


def _round4(n: int) -> int:
    return (n + 3) & ~3


class Engine:
    def __init__(self, model: DecoderModel, runtime: Runtime, config: EngineConfig):
        self.model, self.runtime, self.config = model, runtime, config
        self.kernels = runtime.kernels
        self.vocab_size = model.spec.vocab_size
        self.max_seq_len = min(config.max_seq_len, model.spec.max_positions)
        requests = model.cache_requests()
        num_pages = config.resolved_num_pages()
        if config.num_pages is None and config.gpu_memory_fraction is not None and runtime.device.type == "cuda":
            # as many pages as fit beside what the device already holds (the weights), up to that share of its
            # memory; never more than every slot at full length needs
            free, total = torch.cuda.mem_get_info(runtime.device)
            budget = int(config.gpu_memory_fraction * total) - (total - free)
            per_page = CacheManager.bytes_per_page(requests, config.page_size, runtime.dtype)
            if per_page:
                fit = budget // per_page - 1                      # the scratch page
                if fit < 1:
                    raise ValueError(f"gpu_memory_fraction {config.gpu_memory_fraction} leaves no room for a cache page "
                                     f"({(total - free) >> 20} MiB of {total >> 20} MiB are in use)")
                num_pages = min(num_pages, int(fit))
        self.cache = CacheManager(requests, config.page_size, num_pages,
                                  config.max_batch_size, self.max_seq_len, runtime.device, runtime.dtype)
        self._pinned = runtime.device.type == "cuda"
        self._staging = [None, None]          # two host buffers in turn, each with the event of its last copy
        self._staging_events = [None, None]
        self._staging_turn = 0
        self.h2d_bytes = 0                  # bytes of step inputs copied from the host so far
        self.steps_run = 0
        self.graphs = self.prompt_graphs = None
        if config.cuda_graph and runtime.device.type == "cuda" and model.graph_safe():
            from .graph import DecodeGraphs, PromptGraphs
            self.graphs = DecodeGraphs(self)
            self.prompt_graphs = PromptGraphs(self)

    # ------------------------------------------------------------------ requests
    def admit(self, request_id) -> None:
        self.cache.admit(request_id)

    def finish(self, request_id) -> None:
        """The request is over: what it holds is given back."""
        self.cache.release(request_id)

    def context_length(self, request_id) -> int:
        return self.cache.length(request_id)

    # ------------------------------------------------------------------ the batch
    def _stage(self, count: int) -> torch.Tensor:
        """A pinned host buffer that no copy in flight still reads."""
        self._staging_turn ^= 1
        i = self._staging_turn
        if self._staging_events[i] is not None:
            self._staging_events[i].synchronize()
        if self._staging[i] is None or self._staging[i].numel() < count:
            self._staging[i] = torch.empty(max(count, 4096), dtype=torch.int32, pin_memory=self._pinned)
        return self._staging[i][:count]

    def _record_staging(self) -> None:
        """Mark the point after which the host buffer handed out last may be written again."""
        if self._staging_events[self._staging_turn] is None:
            self._staging_events[self._staging_turn] = torch.cuda.Event()
        self._staging_events[self._staging_turn].record()

    def _to_device(self, host: torch.Tensor) -> torch.Tensor:
        if not self._pinned:
            return host.clone()
        dev = host.to(self.runtime.device, non_blocking=True)
        self.h2d_bytes += host.numel() * host.element_size()
        self._record_staging()
        return dev

    def _fill_host(self, entries: List[StepEntry], pad_to: int = 0, table_width: Optional[int] = None,
                   want_all: bool = False, pad_tokens_to: int = 0):
        """The step's metadata as one packed int32 host buffer. With pad_to, segments of one
        token at position 0 on the scratch page are appended until there are pad_to segments
        (a captured decode step has a fixed number of rows); with pad_tokens_to, one segment that
        brings the step to that many tokens (a captured prompt step has a fixed number of tokens
        in two segments; an entry that fills it alone is followed by a segment of no tokens).
        Returns (host, layout, lists)."""
        cache = self.cache
        seg_lens = [len(e.tokens) for e in entries]
        seg_pos0 = [cache.length(e.request_id) for e in entries]
        seg_slot = [cache.slot(e.request_id) for e in entries]
        real = len(entries)
        pad_lens = [1] * max(0, pad_to - real)
        if pad_tokens_to:
            pad_lens = [pad_tokens_to - sum(seg_lens)]
        pad, pad_tokens = len(pad_lens), sum(pad_lens)
        T, R = sum(seg_lens) + pad_tokens, real + pad
        want_rows, base = [], 0
        for e, n in zip(entries, seg_lens):
            for w in e.want:
                if not 0 <= w < n:
                    raise ValueError(f"request {e.request_id!r}: wanted place {w} is outside its {n} tokens")
                want_rows.append(base + w)
            base += n
        if want_all:
            want_rows = list(range(T))
        N = len(want_rows)
        max_context = max(p + n for p, n in zip(seg_pos0, seg_lens))
        groups = cache.paged_groups()
        W = table_width or max(1, -(-max_context // cache.page_size))

        o_tok, o_pos, o_seg = 0, _round4(T), 2 * _round4(T)
        o_cu = 3 * _round4(T)
        o_p0 = o_cu + _round4(R + 1)
        o_slot = o_p0 + _round4(R)
        o_want = o_slot + _round4(R)
        o_tab = o_want + _round4(max(N, 1))
        seg_lens_all = seg_lens + pad_lens
        pos0_all = seg_pos0 + [0] * pad
        slot_all = seg_slot + [cache.scratch_slot] * pad      # padded rows own no request's state
        # small tables that the mixers' kernels derive from the step's shape travel in the same copy
        step_tables = self.model.step_tables(seg_lens_all, pos0_all, pad_tokens_to)
        o_extra, extras = o_tab + len(groups) * _round4(R * W), []
        for key, table in step_tables.items():
            extras.append((key, o_extra, tuple(table.shape)))
            o_extra += _round4(table.size)
        total = o_extra
        host = self._stage(total)
        buf = host.numpy()
        tokens = np.fromiter((t for e in entries for t in e.tokens), dtype=np.int64, count=T - pad_tokens)
        if tokens.size and (tokens.min() < 0 or tokens.max() >= self.vocab_size):
            raise ValueError(f"a token id lies outside the vocabulary of {self.vocab_size}")
        buf[o_tok:o_tok + T - pad_tokens] = tokens
        buf[o_tok + T - pad_tokens:o_tok + T] = 0
        lens = np.asarray(seg_lens_all, dtype=np.int32)
        cu = np.zeros(R + 1, dtype=np.int32)
        np.cumsum(lens, out=cu[1:])
        seg_ids = np.repeat(np.arange(R, dtype=np.int32), lens)
        pos0 = np.asarray(pos0_all, dtype=np.int32)
        buf[o_seg:o_seg + T] = seg_ids
        buf[o_pos:o_pos + T] = np.arange(T, dtype=np.int32) - cu[:-1][seg_ids] + pos0[seg_ids]
        buf[o_cu:o_cu + R + 1] = cu
        buf[o_p0:o_p0 + R] = pos0
        buf[o_slot:o_slot + R] = slot_all
        buf[o_want:o_want + N] = want_rows
        for i, g in enumerate(groups):
            start = o_tab + i * _round4(R * W)
            buf[start:start + real * W] = cache.table_rows(g, seg_slot, W).reshape(-1)
            buf[start + real * W:start + R * W] = 0
        for (key, start, shape), table in zip(extras, step_tables.values()):
            buf[start:start + table.size] = table.reshape(-1)
        layout = dict(T=T, R=R, N=N, W=W, o_tok=o_tok, o_pos=o_pos, o_seg=o_seg, o_cu=o_cu, o_p0=o_p0, o_slot=o_slot,
                      o_want=o_want, o_tab=o_tab, total=total, groups=groups, extras=extras)
        lists = dict(seg_lens=seg_lens_all, seg_pos0=pos0_all, seg_slot=slot_all, max_context=max_context,
                     wants_every_row=want_rows == list(range(T)))
        return host, layout, lists

    def _batch_from(self, dev: torch.Tensor, layout: dict, lists: dict) -> StepBatch:
        L = layout
        T, R, N, W = L["T"], L["R"], L["N"], L["W"]
        batch = StepBatch(
            num_tokens=T, num_segments=R,
            token_ids=dev[L["o_tok"]:L["o_tok"] + T], positions=dev[L["o_pos"]:L["o_pos"] + T],
            seg_of_token=dev[L["o_seg"]:L["o_seg"] + T], cu_seqlens=dev[L["o_cu"]:L["o_cu"] + R + 1],
            seg_pos0=dev[L["o_p0"]:L["o_p0"] + R], seg_slot=dev[L["o_slot"]:L["o_slot"] + R],
            want_rows=dev[L["o_want"]:L["o_want"] + N], num_wanted=N,
            seg_lens=lists["seg_lens"], seg_pos0_list=lists["seg_pos0"], seg_slot_list=lists["seg_slot"],
            max_seg_len=max(lists["seg_lens"]), max_context=lists["max_context"],
            wants_every_row=lists.get("wants_every_row", False),
        )
        for i, g in enumerate(L["groups"]):
            start = L["o_tab"] + i * _round4(R * W)
            batch.block_tables[g] = dev[start:start + R * W].view(R, W)
        for key, start, shape in L.get("extras", ()):
            count = int(np.prod(shape))
            batch.extras[key] = dev[start:start + count].view(*shape)
        return batch

    def build_batch(self, entries: List[StepEntry], table_width: Optional[int] = None) -> StepBatch:
        """Host lists -> one packed int32 buffer -> one copy to the device -> StepBatch."""
        host, layout, lists = self._fill_host(entries, table_width=table_width)
        return self._batch_from(self._to_device(host), layout, lists)

    # ------------------------------------------------------------------ the step
    def step(self, entries: List[StepEntry], token_feedback: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Run the entries' tokens as one batch. Returns float32 logits [wanted, vocab] on
        the device. Raises OutOfPages (nothing was taken or run) if the pages do not suffice.
        token_feedback: for a step in which every request brings one token, an int32 device tensor
        with those tokens (what the sampler produced for the step before); the ids in the entries
        are then placeholders and the host need not wait for the sampler."""
        if not entries:
            return torch.empty(0, self.vocab_size, dtype=torch.float32, device=self.runtime.device)
        seen = set()
        for e in entries:
            if len(e.tokens) < 1:
                raise ValueError(f"request {e.request_id!r} brings no tokens")
            if e.request_id in seen:
                raise ValueError(f"request {e.request_id!r} appears twice in one step")
            seen.add(e.request_id)
            if min(e.tokens) < 0 or max(e.tokens) >= self.vocab_size:
                raise ValueError(f"request {e.request_id!r}: a token id lies outside the vocabulary of {self.vocab_size}")
            for w in e.want:
                if not 0 <= w < len(e.tokens):
                    raise ValueError(f"request {e.request_id!r}: wanted place {w} is outside its {len(e.tokens)} tokens")
        total = sum(len(e.tokens) for e in entries)
        if total > self.config.max_step_tokens:
            raise ValueError(f"the step holds {total} tokens; the budget is {self.config.max_step_tokens}")
        admitted = []
        try:
            for e in entries:
                if not self.cache.is_live(e.request_id):
                    self.cache.admit(e.request_id)
                    admitted.append(e.request_id)
            for e in entries:
                self.cache.reserve(e.request_id, self.cache.length(e.request_id) + len(e.tokens))
        except Exception:
            for e in entries:                 # nothing of this step stays taken
                if e.request_id in admitted:
                    self.cache.release(e.request_id)
                elif self.cache.is_live(e.request_id):
                    self.cache.trim(e.request_id)
            raise
        if token_feedback is not None and not (self.graphs is not None and total == len(entries)):
            for e in entries:
                self.cache.trim(e.request_id)
            raise ValueError("token_feedback needs a captured decode step: one token per request, cuda_graph on")
        if self.graphs is not None and total == len(entries):
            logits = self.graphs.run(entries, token_feedback)   # one token per request: replay a captured step
        elif self.prompt_graphs is not None and self.prompt_graphs.takes(entries):
            logits = self.prompt_graphs.run(entries)            # a short first portion of one request: likewise
        else:
            batch = self.build_batch(entries)
            logits = self.model.forward(batch, self.cache)
        for e in entries:
            self.cache.commit(e.request_id, self.cache.length(e.request_id) + len(e.tokens))
        self.steps_run += 1
        return logits

    def can_feed_back(self) -> bool:
        """Whether decode steps can take their tokens from the device (captured steps are on)."""
        return self.graphs is not None

    def decode_steps(self, request_ids: List, tokens: List[int], steps: int) -> List[List[int]]:
        """`steps` greedy decode steps for live requests without the host in between: every step
        takes its tokens from the sampler's output of the step before, on the device, and the
        sampled ids travel to pinned host memory behind the steps. Returns tokens[step][request].
        The reference's traced decode feeds tokens and positions back on the device in the same
        way (src/tt_transformers/llm_runtime/decode.py:1137-1140)."""
        rows = len(request_ids)
        if steps <= 0 or rows == 0:
            return []
        if not self.can_feed_back():
            out, cur = [], list(tokens)
            for _ in range(steps):
                logits = self.step([StepEntry(r, [t], [0]) for r, t in zip(request_ids, cur)])
                cur = self.kernels.sample(logits).tolist()
                out.append(cur)
            return out
        from .graph import OWN_ARGMAX

        host = torch.empty(steps, rows, dtype=torch.int32, pin_memory=True)
        feedback, cur = None, list(tokens)
        for s in range(steps):
            self.step([StepEntry(r, [t], [0]) for r, t in zip(request_ids, cur)], token_feedback=feedback)
            host[s].copy_(self.graphs.greedy, non_blocking=True)     # the captured step's own argmax
            feedback = OWN_ARGMAX
            cur = [0] * rows                      # placeholders: the device feeds the real ids
        torch.cuda.current_stream(self.runtime.device).synchronize()
        return host.tolist()

    def warmup(self, batch_sizes=None, context_buckets=None, prompts: bool = True) -> int:
        """Capture ahead of time what would otherwise be captured at first use, so that no request waits for a
        capture: decode steps for every captured batch size (or those given) and context bucket (or those given),
        and the prompt steps of every length bucket. Needs an engine without live requests; takes pages for as
        many one-token requests as the largest batch size and gives them back. Returns how many steps were
        captured. The reference warms its traces up in the same way before serving
        (src/tt_transformers/llm_runtime/config.py:18-75, WarmupConfig)."""
        if self.graphs is None:
            return 0
        if self.cache.live_requests():
            raise RuntimeError("warmup() wants an engine without live requests")
        graphs, captured = self.graphs, 0
        sizes = [s for s in (batch_sizes or graphs.sizes) if s <= self.config.max_batch_size]
        if context_buckets is None:
            context_buckets, bucket = [], graphs.MIN_CONTEXT_BUCKET
            while bucket < self.max_seq_len:
                context_buckets.append(bucket)
                bucket *= 2
            context_buckets.append(self.max_seq_len)
        context_buckets = sorted({min(b, self.max_seq_len) for b in context_buckets})
        ids = [("warmup", i) for i in range(max(sizes, default=0))]
        try:
            for rid in ids:
                self.cache.admit(rid)
                self.cache.reserve(rid, 1)
            for size in sizes:
                entries = [StepEntry(rid, [0], [0]) for rid in ids[:size]]
                for bucket in context_buckets:
                    if (size, bucket) not in graphs._graphs:
                        graphs._graphs[(size, bucket)] = graphs._capture(size, bucket, entries)
                        captured += 1
        finally:
            for rid in ids:
                if self.cache.is_live(rid):
                    self.cache.release(rid)
        if prompts and self.prompt_graphs is not None:
            for size in self.prompt_graphs.sizes:
                if size in self.prompt_graphs._graphs:
                    continue
                rid = ("warmup", "prompt")
                self.cache.admit(rid)
                try:
                    self.cache.reserve(rid, 2)
                    self.prompt_graphs._graphs[size] = self.prompt_graphs._capture(size, [StepEntry(rid, [0, 0], [1])])
                    captured += 1
                finally:
                    self.cache.release(rid)
        torch.cuda.synchronize(self.runtime.device)
        return captured

    def close(self) -> None:
        for rid in self.cache.live_requests():
            self.cache.release(rid)
        for g in self.cache.groups:
            g.storage = None                     # the pages and the state tensors go
        self.graphs = self.prompt_graphs = None


def build_engine(model_folder: str = None, engine_config: EngineConfig = None, *, config_dict: dict = None,
                 tensors: Dict[str, torch.Tensor] = None, kernels=None, n_layers: int = None) -> Engine:
    """From a model folder (config.json + safetensors), or from a configuration dictionary
    and tensors held in memory, to an engine ready to step. The model class is chosen by
    config.json's `architectures`. `kernels` None loads the CUDA kernel table of the
    engine's device; there is no other implementation in this package."""
    engine_config = engine_config or EngineConfig()
    if model_folder is not None:
        config_dict = read_config_json(model_folder)
    elif config_dict is None or tensors is None:
        raise ValueError("give a model folder, or config_dict and tensors")
    arch = get_architecture(architecture_of(config_dict))
    cfg = arch.load_config(config_dict)
    spec = arch.model_spec(cfg)
    if n_layers is not None:
        spec = spec.first_entries(n_layers)       # the model cut short, whatever the architecture
    model = DecoderModel(spec)
    specs = model.tensor_specs()
    if model_folder is not None:
        tensors = read_safetensors(model_folder, wanted=[s.name for s in specs] if n_layers is not None else None,
                                   widen_float16=engine_config.dtype == "float32")
    if n_layers is not None:
        # a model cut to its first layers leaves the other layers' tensors unused on purpose
        check_tensors(tensors, specs, ignorable=lambda name: True)
    else:
        check_tensors(tensors, specs, ignorable=lambda name: arch.ignorable(cfg, name))
    device = torch.device(engine_config.device)
    if kernels is None:
        from ..kernels import load_kernels
        kernels = load_kernels(device)
    runtime = Runtime(kernels=kernels, device=device, dtype=_DTYPES[engine_config.dtype])
    model.bind(tensors, runtime)
    engine = Engine(model, runtime, engine_config)
    engine.model_config = cfg
    return engine
