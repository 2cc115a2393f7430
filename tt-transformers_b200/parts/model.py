"""A decoder model as data, and the generic model that runs it.

`ModelSpec` names the parts of every layer (kind + parameters), the order in which
layers run, and the embedding, final norm and head. `DecoderModel` builds the parts
from the registries and runs a step. An architecture is a function from its typed
configuration to a ModelSpec; nothing here knows any architecture.

The layer order is a list of `LayerCall`s. A call names the layer to run; by default
it owns a cache unit of its own. `cache_of=j` makes it read (never write) the unit of
the j-th call instead. A layer may be named by several calls (shared weights).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from .base import ADDED, DeferredNorm, PartSpec, Runtime, StepBatch, TensorSpec, build_part
from .embedding import Embedding, Head


@dataclass(frozen=True)
class LayerSpec:
    mixer: PartSpec
    feed_forward: PartSpec
    norm1: PartSpec
    norm2: PartSpec
    position: Optional[PartSpec] = None      # handed to the mixer as `position`
    block: str = "pre_norm"


@dataclass(frozen=True)
class LayerCall:
    layer: int
    cache_of: Optional[int] = None           # index into the layer order, earlier than this call


@dataclass(frozen=True)
class ModelSpec:
    vocab_size: int
    width: int
    embedding_name: str
    layers: tuple                            # of LayerSpec
    order: tuple                             # of LayerCall
    final_norm: PartSpec
    head_name: Optional[str]                 # None: tied to the embedding
    input_position: Optional[PartSpec] = None  # a position encoding applied to the embedded tokens
    max_positions: int = 1 << 30


class DecoderModel:
    def __init__(self, spec: ModelSpec):
        self.spec = spec
        self.embedding = Embedding(spec.vocab_size, spec.width, spec.embedding_name)
        self.head = Head(spec.vocab_size, spec.width, spec.head_name,
                         tied_to=self.embedding if spec.head_name is None else None)
        self.final_norm = build_part("norm", spec.final_norm)
        self.input_position = build_part("position", spec.input_position) if spec.input_position else None
        self.layers = []
        positions: Dict[PartSpec, object] = {}
        for ls in spec.layers:
            position = None
            if ls.position is not None:
                if ls.position not in positions:          # layers with the same encoding share one object
                    positions[ls.position] = build_part("position", ls.position)
                position = positions[ls.position]
            mixer_params = dict(ls.mixer.params)
            if position is not None:
                mixer_params["position"] = position
            mixer = build_part("mixer", PartSpec(ls.mixer.kind, mixer_params))
            block = build_part("block", PartSpec(ls.block, dict(
                norm1=build_part("norm", ls.norm1), mixer=mixer,
                norm2=build_part("norm", ls.norm2), feed_forward=build_part("feed_forward", ls.feed_forward))))
            self.layers.append(block)
        self.positions = list(positions.values())
        for i, call in enumerate(spec.order):
            if not 0 <= call.layer < len(self.layers):
                raise ValueError(f"layer order entry {i} names layer {call.layer}, which does not exist")
            if call.cache_of is not None and not (0 <= call.cache_of < i and spec.order[call.cache_of].cache_of is None):
                raise ValueError(f"layer order entry {i}: cache_of must name an earlier entry that owns its cache")

    # ------------------------------------------------------------------ weights
    def all_parts(self):
        parts = [self.embedding, self.head, self.final_norm]
        if self.input_position is not None:
            parts.append(self.input_position)
        parts.extend(self.positions)
        for block in self.layers:
            parts.extend(block.parts())
        return parts

    def tensor_specs(self) -> List[TensorSpec]:
        seen, out = set(), []
        for part in self.all_parts():
            for spec in part.tensor_specs():
                if spec.name not in seen:
                    seen.add(spec.name)
                    out.append(spec)
        return out

    def bind(self, tensors: Dict[str, torch.Tensor], runtime: Runtime) -> None:
        self.runtime = runtime
        for part in self.all_parts():
            part.bind(tensors, runtime)

    def graph_safe(self) -> bool:
        """True if every mixer and feed-forward says that its forward only launches kernels
        on the current stream with shapes fixed by the batch's shape (no host reads, no
        per-step host tables), so that a decode step may be captured and replayed."""
        return all(getattr(p, "graph_safe", False) for b in self.layers for p in (b.mixer, b.feed_forward))

    # ------------------------------------------------------------------ cache needs
    def cache_requests(self):
        """For every entry of the layer order: what its cache unit must be (PagedKV,
        SlotState or None), or the index of the entry whose unit it reads."""
        out = []
        for call in self.spec.order:
            if call.cache_of is not None:
                out.append(call.cache_of)
            else:
                out.append(self.layers[call.layer].mixer.cache_request())
        return out

    # ------------------------------------------------------------------ one step
    def forward(self, batch: StepBatch, cache) -> torch.Tensor:
        """Run the step's tokens; `cache.view(entry, batch)` gives each entry's cache view.
        Returns float32 logits [num_wanted, vocab]."""
        k = self.runtime.kernels
        x = self.embedding.forward(batch.token_ids)
        if self.input_position is not None:
            x = self.input_position.embed(x, batch)
        delta = None
        order = self.spec.order
        for i, call in enumerate(order):
            owner = i if call.cache_of is None else call.cache_of
            block = self.layers[call.layer]
            view = cache.view(owner, batch)
            if getattr(block, "takes_next_norm", False):
                # the norm that will run on this block's result, if what follows it can take it half done
                if i + 1 < len(order):
                    nxt = self.layers[order[i + 1].layer]
                    norm, consumer = getattr(nxt, "norm1", None), getattr(nxt, "mixer", None)
                else:
                    norm, consumer = self.final_norm, self.head
                    if not batch.wants_every_row:
                        norm = None              # the head sees a selection of the rows
                ok = (norm is not None and getattr(norm, "can_defer", False) and getattr(consumer, "fuses_norm", False))
                x, delta = block.forward(x, delta, batch, view, write_cache=call.cache_of is None,
                                         next_norm=norm if ok else None)
            else:
                if delta is ADDED or isinstance(delta, DeferredNorm):
                    delta = None
                x, delta = block.forward(x, delta, batch, view, write_cache=call.cache_of is None)
        if batch.num_wanted == 0:
            return torch.empty(0, self.spec.vocab_size, dtype=torch.float32, device=x.device)
        if isinstance(delta, DeferredNorm) and delta.made_for is self.final_norm and batch.wants_every_row:
            return self.head.forward(self.final_norm.forward_add(x, delta, defer=True))
        if delta is ADDED or isinstance(delta, DeferredNorm):
            delta = None
        if not batch.wants_every_row:
            x = k.gather_rows(x, batch.want_rows)
            if delta is not None:
                delta = k.gather_rows(delta, batch.want_rows)
        h = self.final_norm.forward_add(x, delta)
        return self.head.forward(h)
