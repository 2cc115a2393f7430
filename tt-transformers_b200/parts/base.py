"""What a part is, what it may ask of the cache, and where parts are registered.

A part (mixer, feed-forward, norm, position encoding, embedding, head) is built
from a kind name and a dictionary of parameters: all of its sizes and constants.
It declares the checkpoint tensors it needs, takes them at `bind`, and then runs
on the tensors of one step. No part knows which model it is in; the reference
builds its modules the same way, from explicit weights and dimensions
(src/tt_transformers/modules/README.md:18-31,40-66).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

import torch


# ----------------------------------------------------------------------------- tensors a part needs
@dataclass(frozen=True)
class TensorSpec:
    """One checkpoint tensor: its full name, its shape, and whether it holds
    floating-point values ("float") or an integer table ("int")."""

    name: str
    shape: Tuple[int, ...]
    kind: str = "float"
    optional: bool = False


# ----------------------------------------------------------------------------- what a mixer asks of the cache
@dataclass(frozen=True)
class PagedKV:
    """Keys and values in pages. `window` None keeps all keys; a number keeps only
    the last `window` positions readable, and pages behind it are given back."""

    num_kv_heads: int
    head_dim: int
    window: Optional[int] = None


@dataclass(frozen=True)
class SlotState:
    """A tensor of fixed shape per live request (float32), zeroed when the request
    is admitted. Mixers with a running state of their own use this."""

    shape: Tuple[int, ...]


@dataclass
class PagedKVView:
    """One cache unit of a paged group as a mixer sees it during a step."""

    keys: torch.Tensor          # [num_pages, kv_heads, page_size, head_dim]
    values: torch.Tensor        # same shape
    block_table: torch.Tensor   # int32 [segments, pages_per_request]; entry i covers positions i*page_size ..
    page_size: int
    window: Optional[int]


@dataclass
class SlotStateView:
    state: torch.Tensor         # [max_slots, *shape] float32
    slots: torch.Tensor         # int32 [segments] on the device
    slot_list: List[int]        # the same on the host


# ----------------------------------------------------------------------------- what every part is given
@dataclass
class Runtime:
    """Where and how parts compute: the kernel table, the device, the compute dtype."""

    kernels: object
    device: torch.device
    dtype: torch.dtype          # torch.bfloat16 or torch.float32

    def matrix(self, tensor: torch.Tensor) -> torch.Tensor:
        """A matrix operand on the device in the compute dtype."""
        return tensor.to(device=self.device, dtype=self.dtype).contiguous()

    def vector(self, tensor: torch.Tensor) -> torch.Tensor:
        """A small per-channel vector: a tensor stored in 32-bit stays so, others
        take the compute dtype."""
        dtype = torch.float32 if tensor.dtype == torch.float32 else self.dtype
        return tensor.to(device=self.device, dtype=dtype).contiguous()


@dataclass
class StepBatch:
    """The tokens of one step, flat: segment r owns tokens cu_seqlens[r] ..
    cu_seqlens[r+1]. Device tensors are int32; the host lists mirror them."""

    num_tokens: int
    num_segments: int
    token_ids: torch.Tensor       # [T]
    positions: torch.Tensor       # [T] absolute position of each token in its request
    seg_of_token: torch.Tensor    # [T]
    cu_seqlens: torch.Tensor      # [R+1]
    seg_pos0: torch.Tensor        # [R] tokens of the request cached before this step
    seg_slot: torch.Tensor        # [R]
    want_rows: torch.Tensor       # [N] flat token indices whose logits are wanted
    num_wanted: int
    seg_lens: List[int] = field(default_factory=list)
    seg_pos0_list: List[int] = field(default_factory=list)
    seg_slot_list: List[int] = field(default_factory=list)
    max_seg_len: int = 1
    max_context: int = 1          # the largest pos0 + len over the segments
    wants_every_row: bool = False  # want_rows is 0, 1, .. num_tokens-1
    block_tables: Dict[int, torch.Tensor] = field(default_factory=dict)  # group index -> [R, W]
    extras: dict = field(default_factory=dict)   # per-step tables that kernels derive once and reuse in every layer


class DeferredNorm:
    """A norm whose scaling is still to come. The product that ended the sub-layer before it has
    left `xg` = compute-dtype(g * residual) [rows, width], g being the norm's weight, and `ssq`
    [parts, 16] float32, partial sums of residual^2 per row; the norm's output is
    xg / sqrt(sum(ssq) / width + eps). A skinny matrix product takes this in place of the normalised
    tensor (it divides its sums instead of its input); everything else calls materialize().
    `made_for`: the norm part whose weight and eps went in."""

    __slots__ = ("xg", "ssq", "eps", "made_for", "_materialize")

    def __init__(self, xg, ssq, eps, made_for, materialize):
        self.xg, self.ssq, self.eps, self.made_for, self._materialize = xg, ssq, float(eps), made_for, materialize

    @property
    def shape(self):
        return self.xg.shape

    def materialize(self):
        return self._materialize()


class _Added:
    """What a part returns instead of its output when it has already added that output to the
    residual stream it was given."""

    def __repr__(self):
        return "ADDED"


ADDED = _Added()


class Part:
    """Base of all parts. Two optional capabilities, off unless a part says otherwise:
    `fuses_norm`: forward() accepts a DeferredNorm in place of x; `fuses_residual`: forward()
    accepts residual=<float32 stream> and next_norm=<the norm part that follows, or None>, may add
    its output to the stream itself and then returns ADDED, or a DeferredNorm made for next_norm."""

    fuses_norm = False
    fuses_residual = False

    def tensor_specs(self) -> List[TensorSpec]:
        return []

    def bind(self, tensors: Dict[str, torch.Tensor], runtime: Runtime) -> None:
        self.runtime = runtime


class Mixer(Part):
    """Mixes information between the positions of a request.

    forward(x [T, width], batch, cache, write_cache) -> [T, width].
    `cache` is the view that matches cache_request(): PagedKVView, SlotStateView or
    None. With write_cache False the unit belongs to an earlier entry of the
    layer order and must only be read.
    """

    def cache_request(self):
        return None

    def forward(self, x, batch: StepBatch, cache, write_cache: bool = True):
        raise NotImplementedError


class FeedForward(Part):
    """forward(x [T, width], batch) -> [T, width], each token by itself."""

    def forward(self, x, batch: StepBatch):
        raise NotImplementedError


class Norm(Part):
    """forward_add(residual, delta) adds delta (or nothing, if None) into the
    float32 residual stream in place and returns the normalised tensor in the
    compute dtype. delta may be ADDED (nothing left to add). A norm with `can_defer`
    has fusion_args() -> (float32 weight, eps), accepts a DeferredNorm made for it as delta and,
    with defer=True, may hand it on instead of a tensor."""

    can_defer = False

    def forward_add(self, residual, delta):
        raise NotImplementedError


class PositionEncoding(Part):
    """How positions reach the model. `embed` may change the embedded tokens
    (absolute encodings); `rotation()` gives what a mixer needs to rotate queries
    and keys: (inverse frequencies float32 [rotary_dim/2] on the device,
    rotary_dim), or None when nothing is rotated."""

    def embed(self, x, batch: StepBatch):
        return x

    def rotation(self):
        return None


# ----------------------------------------------------------------------------- registries
_REGISTRIES: Dict[str, Dict[str, Callable]] = {
    "mixer": {}, "feed_forward": {}, "norm": {}, "position": {}, "block": {},
}


def register_part(category: str, kind: str, factory: Callable) -> None:
    """Make `factory(**params)` available as `kind` in `category` (mixer,
    feed_forward, norm, position, block). Registering a kind again replaces it."""
    if category not in _REGISTRIES:
        raise KeyError(f"unknown part category {category!r}; known: {sorted(_REGISTRIES)}")
    _REGISTRIES[category][kind] = factory


def build_part(category: str, spec: "PartSpec"):
    table = _REGISTRIES[category]
    if spec.kind not in table:
        raise KeyError(f"no {category} of kind {spec.kind!r} is registered; known: {sorted(table)}")
    return table[spec.kind](**spec.params)


@dataclass(frozen=True)
class PartSpec:
    """A part as data: which kind, and its parameters (sizes, constants, tensor name prefix)."""

    kind: str
    params: dict = field(default_factory=dict)

    def __hash__(self):
        return hash((self.kind, tuple(sorted((k, repr(v)) for k, v in self.params.items()))))
