"""Token embedding and the output head, as registered parts like the others.

Embedding kind `table`: x[t] = scale * E[token[t]]; the reference's embedding module takes the same
`embed_scale` parameter and Llama passes 1 (src/tt_transformers/modules/embedding/embedding_1d.py:140-150).
Head kind `linear`: logits = h W^T in float32, W being the embedding table itself when the checkpoint
ties them (src/tt_transformers/models/llama32_1b/hf_generator.py:254-261; float32 logits:
src/tt_transformers/llm_runtime/decode.py:936-947); optional `scale` on the logits and `logit_cap`
(logits = cap * tanh(logits / cap)), both off for Llama.
"""

from __future__ import annotations

from typing import Optional

import torch

from .base import OutputHead, TensorSpec, TokenEmbedding, register_part


class TableEmbedding(TokenEmbedding):
    def __init__(self, vocab: int, width: int, weight_name: str, scale: float = 1.0):
        self.vocab, self.width, self.weight_name, self.scale = int(vocab), int(width), weight_name, float(scale)

    def tensor_specs(self):
        return [TensorSpec(self.weight_name, (self.vocab, self.width))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.table = runtime.matrix(tensors[self.weight_name])

    def forward(self, token_ids):
        return self.runtime.kernels.embedding(self.table, token_ids, self.scale)


class LinearHead(OutputHead):
    """`weight_name` None: the head shares the table of the embedding it is tied to."""

    fuses_norm = True

    def __init__(self, vocab: int, width: int, weight_name: Optional[str] = None, scale: float = 1.0,
                 logit_cap: Optional[float] = None):
        self.vocab, self.width, self.weight_name = int(vocab), int(width), weight_name
        self.scale = float(scale)
        self.logit_cap = None if logit_cap is None else float(logit_cap)
        if self.logit_cap is not None and not self.logit_cap > 0:
            raise ValueError(f"logit_cap must be positive, got {logit_cap}")
        self.tied = weight_name is None
        self._embedding = None

    def tie(self, embedding: TokenEmbedding) -> None:
        self._embedding = embedding

    def tensor_specs(self):
        if self.tied:
            return []
        return [TensorSpec(self.weight_name, (self.vocab, self.width))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        if self.tied:
            if self._embedding is None or not hasattr(self._embedding, "table"):
                raise ValueError("a head without a weight of its own needs an embedding with a `table` to share")
            self.weight = self._embedding.table        # bound before the head: same storage
        else:
            self.weight = runtime.matrix(tensors[self.weight_name])

    def forward(self, h):
        k = self.runtime.kernels
        logits = k.linear(h, self.weight, out_dtype=torch.float32)
        if self.scale != 1.0:
            logits.mul_(self.scale)
        if self.logit_cap is not None:
            k.softcap(logits, self.logit_cap)
        return logits


register_part("embedding", "table", TableEmbedding)
register_part("head", "linear", LinearHead)
