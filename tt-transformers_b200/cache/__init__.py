"""The cache manager: pages of keys and values, block tables, and per-request slots."""

from .manager import CacheManager, OutOfPages, OutOfSlots
from .pages import PagePool

__all__ = ["CacheManager", "OutOfPages", "OutOfSlots", "PagePool"]
