"""Parts that layers are put together from, and the generic decoder that runs them."""

from . import attention, block, feed_forward, norm, position  # noqa: F401  (they register themselves)
from .base import (FeedForward, Mixer, Norm, PagedKV, PagedKVView, Part, PartSpec, PositionEncoding, Runtime,
                   SlotState, SlotStateView, StepBatch, TensorSpec, build_part, register_part)
from .model import DecoderModel, LayerCall, LayerSpec, ModelSpec

__all__ = ["FeedForward", "Mixer", "Norm", "PagedKV", "PagedKVView", "Part", "PartSpec", "PositionEncoding",
           "Runtime", "SlotState", "SlotStateView", "StepBatch", "TensorSpec", "build_part", "register_part",
           "DecoderModel", "LayerCall", "LayerSpec", "ModelSpec"]
