"""RMSNorm: y = x / sqrt(mean(x^2) + eps) * w, fused with the residual add before it.

Formula: src/tt_transformers/modules/rmsnorm/rmsnorm_1d.py:208-215 (no unit offset,
:68); statistics in float32 (:346-354). Here the sum of residual and delta is float32
as well and is written back to the residual stream.
"""

from __future__ import annotations

from .base import DeferredNorm, Norm, TensorSpec, register_part


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

    def forward_add(self, residual, delta, defer=False):
        """defer: the caller's next step can take the norm into its own kernel. With nothing to add
        and rows few enough for such a kernel, no kernel runs here."""
        k = self.runtime.kernels
        if defer and delta is None and getattr(k, "defers_norm", None) and k.defers_norm(residual, self.runtime.dtype):
            if self._weight_f32 is None:
                self._weight_f32 = self.weight.float().contiguous()
            return DeferredNorm(residual, self._weight_f32, self.eps,
                                lambda: k.add_rmsnorm(residual, None, self.weight, self.eps, self.runtime.dtype))
        return k.add_rmsnorm(residual, delta, self.weight, self.eps, self.runtime.dtype)


register_part("norm", "rmsnorm", RMSNorm)
