"""hayate_b200: B200-native paged-KV attention path for the hayate engine.

Drop-in for ``hayate.engine.paged_cache``: ``PagedKVCacheManager.begin_batch``
returns a batch whose ``write_layer``/``attend_layer`` run hand-written sm_100a
kernels (page-table KV scatter, tcgen05 chunked prefill, split-KV decode)
through the C ABI of ``libhayate_b200.so``.
"""

from .cache import Cache, KVSnapshot
from .paged_cache import (
    MIN_KV_PAGE_SIZE,
    PagedCacheHandle,
    PagedKVBatch,
    PagedKVCacheManager,
)
from .prefix_cache import PagedPrefixCache, PrefixCacheMatch
from . import ops

__all__ = [
    "Cache",
    "KVSnapshot",
    "MIN_KV_PAGE_SIZE",
    "PagedCacheHandle",
    "PagedKVBatch",
    "PagedKVCacheManager",
    "PagedPrefixCache",
    "PrefixCacheMatch",
    "ops",
]
