"""RMSNorm: y = x / sqrt(mean(x^2) + eps) * w, fused with the residual add before it.

Formula: src/tt_transformers/modules/rmsnorm/rmsnorm_1d.py:208-215 (no unit offset,
:68); statistics in float32 (:346-354). Here the sum of residual and delta is float32
as well and is written back to the residual stream.
"""

from __future__ import annotations

from .base import ADDED, DeferredNorm, Norm, TensorSpec, register_part


class RMSNorm(Norm):
    can_defer = True

    def __init__(self, width: int, eps: float, weight_name: str):
        self.width, self.eps, self.weight_name = int(width), float(eps), weight_name

    def tensor_specs(self):
        return [TensorSpec(self.weight_name, (self.width,))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.weight = runtime.vector(tensors[self.weight_name])
        self._weight_f32 = None

    def fusion_args(self):
        """What a product needs to prepare this norm in its epilogue: the weight in float32 and eps."""
        if self._weight_f32 is None:
            self._weight_f32 = self.weight.float().contiguous()
        return self._weight_f32, self.eps

    def forward_add(self, residual, delta, defer=False):
        """defer: the caller's next step takes a DeferredNorm. If the sub-layer before has prepared this
        norm (delta is a DeferredNorm made for it), no kernel runs here."""
        k = self.runtime.kernels
        if isinstance(delta, DeferredNorm):
            if delta.made_for is self:
                return delta if defer else delta.materialize()
            delta = None                         # prepared for another norm: the stream itself is up to date
        if delta is ADDED:
            delta = None
        return k.add_rmsnorm(residual, delta, self.weight, self.eps, self.runtime.dtype)


register_part("norm", "rmsnorm", RMSNorm)
