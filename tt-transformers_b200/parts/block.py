"""How norm, mixer and feed-forward are arranged in one layer.

`pre_norm`: h = norm(x); x = x + mixer(h); h = norm(x); x = x + ff(h)
(src/tt_transformers/models/llama32_1b/model.py:113-139,141-186). The residual stream x
is float32. A sub-layer's output is not added at once: it is handed on as `delta` and
added inside the next norm kernel, which reads and writes x once instead of twice.

Parts that say so fuse further: a sub-layer with `fuses_residual` is given the stream and the norm
that follows, and may add its output to the stream itself (its last product's epilogue does it)
and prepare that norm on the way (ADDED or a DeferredNorm comes back); a norm with `can_defer`
before a sub-layer with `fuses_norm` hands the DeferredNorm on, and that sub-layer's first product
finishes it. A decode layer then runs no norm kernel at all. Parts without these flags see
tensors only, as before.
"""

from __future__ import annotations

from .base import ADDED, Block, DeferredNorm, register_part


def _normed(norm, consumer, x, delta):
    if getattr(norm, "can_defer", False):
        return norm.forward_add(x, delta, defer=bool(getattr(consumer, "fuses_norm", False)))
    if delta is ADDED or isinstance(delta, DeferredNorm):
        delta = None                             # the stream is up to date; this norm knows tensors only
    return norm.forward_add(x, delta)


def _following(norm, consumer):
    """The norm to prepare in a sub-layer's last product: only one that can take it, before a part that can."""
    if norm is not None and getattr(norm, "can_defer", False) and getattr(consumer, "fuses_norm", False):
        return norm
    return None


class PreNormBlock(Block):
    slots = {"norm1": "norm", "mixer": "mixer", "norm2": "norm", "feed_forward": "feed_forward"}
    takes_next_norm = True

    def __init__(self, norm1, mixer, norm2, feed_forward):
        self.norm1, self.mixer, self.norm2, self.feed_forward = norm1, mixer, norm2, feed_forward

    def forward(self, x, delta, batch, cache, write_cache=True, next_norm=None):
        """x: float32 residual, updated in place; delta: pending sub-layer output, None, or ADDED
        (nothing pending) or a DeferredNorm made for norm1. next_norm: the norm that the caller will
        run on the result, if what follows it can take a DeferredNorm. Returns (x, delta)."""
        h = _normed(self.norm1, self.mixer, x, delta)
        if getattr(self.mixer, "fuses_residual", False):
            mixed = self.mixer.forward(h, batch, cache, write_cache, residual=x,
                                       next_norm=_following(self.norm2, self.feed_forward))
        else:
            mixed = self.mixer.forward(h, batch, cache, write_cache)
        h = _normed(self.norm2, self.feed_forward, x, mixed)
        if getattr(self.feed_forward, "fuses_residual", False):
            return x, self.feed_forward.forward(h, batch, residual=x, next_norm=next_norm)
        return x, self.feed_forward.forward(h, batch)


register_part("block", "pre_norm", PreNormBlock)
