"""How norm, mixer and feed-forward are arranged in one layer.

`pre_norm`: h = norm(x); x = x + mixer(h); h = norm(x); x = x + ff(h)
(src/tt_transformers/models/llama32_1b/model.py:113-139,141-186). The residual stream x
is float32. A sub-layer's output is not added at once: it is handed on as `delta` and
added inside the next norm kernel, which reads and writes x once instead of twice.
"""

from __future__ import annotations

from .base import register_part


class PreNormBlock:
    def __init__(self, norm1, mixer, norm2, feed_forward):
        self.norm1, self.mixer, self.norm2, self.feed_forward = norm1, mixer, norm2, feed_forward

    def parts(self):
        return [self.norm1, self.mixer, self.norm2, self.feed_forward]

    def forward(self, x, delta, batch, cache, write_cache=True):
        """x: float32 residual, updated in place; delta: pending sub-layer output or None.
        Returns (x, delta) for the next block."""
        h = self.norm1.forward_add(x, delta)
        mixed = self.mixer.forward(h, batch, cache, write_cache)
        h = self.norm2.forward_add(x, mixed)
        return x, self.feed_forward.forward(h, batch)


register_part("block", "pre_norm", PreNormBlock)
