"""Token embedding and the output head.

Embedding: x[t] = E[token[t]], no scale (src/tt_transformers/modules/embedding/embedding_1d.py:140-150).
Head: logits = h W^T, W being the embedding table itself when the checkpoint ties
them (src/tt_transformers/models/llama32_1b/hf_generator.py:254-261); the logits
leave in float32 (src/tt_transformers/llm_runtime/decode.py:936-947).
"""

from __future__ import annotations

import torch

from .base import Part, TensorSpec


class Embedding(Part):
    def __init__(self, vocab: int, width: int, weight_name: str):
        self.vocab, self.width, self.weight_name = int(vocab), int(width), weight_name

    def tensor_specs(self):
        return [TensorSpec(self.weight_name, (self.vocab, self.width))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.table = runtime.matrix(tensors[self.weight_name])

    def forward(self, token_ids):
        return self.runtime.kernels.embedding(self.table, token_ids)


class Head(Part):
    """`weight_name` None: the head shares the table of `tied_to` (an Embedding)."""

    fuses_norm = True

    def __init__(self, vocab: int, width: int, weight_name=None, tied_to: Embedding = None):
        self.vocab, self.width, self.weight_name, self.tied_to = int(vocab), int(width), weight_name, tied_to
        if (weight_name is None) == (tied_to is None):
            raise ValueError("a head has either a weight of its own or an embedding it is tied to")

    def tensor_specs(self):
        if self.weight_name is None:
            return []
        return [TensorSpec(self.weight_name, (self.vocab, self.width))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.weight = self.tied_to.table if self.weight_name is None else runtime.matrix(tensors[self.weight_name])

    def forward(self, h):
        return self.runtime.kernels.linear(h, self.weight, out_dtype=torch.float32)
