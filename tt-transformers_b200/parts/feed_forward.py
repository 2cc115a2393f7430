"""SwiGLU feed-forward: (silu(x W1) * (x W3)) W2, no biases.

src/tt_transformers/modules/mlp/mlp_1d.py:240-294; tests/modules/mlp/test_mlp_1d.py:676.
Gate (W1) and up (W3) are stacked into one matrix so that one product reads x once.
"""

from __future__ import annotations

import torch

from .base import FeedForward, TensorSpec, register_part


class SwiGLU(FeedForward):
    graph_safe = True

    def __init__(self, width: int, inter: int, prefix: str):
        self.width, self.inter, self.prefix = int(width), int(inter), prefix

    def tensor_specs(self):
        p = self.prefix
        return [TensorSpec(p + "gate_proj.weight", (self.inter, self.width)),
                TensorSpec(p + "up_proj.weight", (self.inter, self.width)),
                TensorSpec(p + "down_proj.weight", (self.width, self.inter))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        self.w_gate_up = runtime.matrix(torch.cat([tensors[p + "gate_proj.weight"], tensors[p + "up_proj.weight"]], 0))
        self.w_down = runtime.matrix(tensors[p + "down_proj.weight"])

    fuses_norm = True
    fuses_residual = True

    def forward(self, x, batch, residual=None, next_norm=None):
        k = self.runtime.kernels
        h = k.linear_swiglu(x, self.w_gate_up)
        if residual is not None:
            # ADDED or a DeferredNorm where the product's epilogue takes the add, else the product itself
            return k.linear(h, self.w_down, accumulate=residual, next_norm=next_norm)
        return k.linear(h, self.w_down)


register_part("feed_forward", "swiglu", SwiGLU)
