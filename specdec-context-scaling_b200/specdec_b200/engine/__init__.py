"""Paged KV cache, the spec_cache contract, and the batched SpecDec engine."""

from .paged_cache import PagedKVCache
from .spec_cache import cache_length, check_consistent, trim_cache, trim_cache_device

__all__ = ["PagedKVCache", "cache_length", "check_consistent", "trim_cache", "trim_cache_device"]
