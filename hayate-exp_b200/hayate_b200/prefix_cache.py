"""Prefix cache that shares physical KV pages instead of copying them.

Same interface and LRU policy as hayate's ``PrefixCache``
(``hayate/engine/prefix_cache.py:18-100``): ``get(tokens, max_prefix_len)``
returns the longest cached prefix, ``put(tokens, source)`` stores one within a
token budget (least recently used entries are evicted first), ``clear()`` drops
everything. The difference is what an entry holds: the reference clones a
contiguous K/V snapshot on ``put`` and copies it back into fresh pages on a hit
(``paged_cache.py:153-190``); here an entry is a page-aliasing handle
(``PagedKVCacheManager.share``), so ``put`` and a hit cost no K/V traffic at all
and a hit's pages are shared until the new request writes into them.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass
from typing import Sequence

from .paged_cache import PagedCacheHandle, PagedKVCacheManager


@dataclass(frozen=True)
class PrefixCacheMatch:
    """Cached token count and a fresh request handle aliasing those tokens' pages."""

    length: int
    handle: PagedCacheHandle | None


class PagedPrefixCache:
    """LRU map from token prefixes to page-aliasing handles of one manager."""

    def __init__(self, manager: PagedKVCacheManager, max_tokens: int):
        if max_tokens < 0:
            raise ValueError("prefix cache token budget must be non-negative")
        self.manager = manager
        self.max_tokens = max_tokens
        self.total_tokens = 0
        self._entries: OrderedDict[tuple[int, ...], PagedCacheHandle] = OrderedDict()

    def get(self, tokens: Sequence[int], max_prefix_len: int | None = None) -> PrefixCacheMatch:
        """Longest cached prefix of ``tokens``; on a hit a NEW handle shares its pages.

        The caller owns the returned handle (release it like any other request).
        """
        if self.max_tokens == 0 or not tokens or not self._entries:
            return PrefixCacheMatch(0, None)
        key = tuple(tokens)
        limit = len(key) if max_prefix_len is None else min(len(key), max_prefix_len)
        if limit <= 0:
            return PrefixCacheMatch(0, None)
        best, best_len = None, 0
        for cached, handle in self._entries.items():
            n = _common_prefix(key, cached, limit)
            if n > best_len and n <= handle.length:
                best, best_len = cached, n
                if best_len == limit:
                    break
        if best is None:
            return PrefixCacheMatch(0, None)
        self._entries.move_to_end(best)
        return PrefixCacheMatch(best_len, self.manager.share(self._entries[best], best_len))

    def put(self, tokens: Sequence[int], source: PagedCacheHandle) -> None:
        """Remember ``tokens``' prefix as held by ``source`` (aliases its pages, no copy)."""
        if self.max_tokens == 0 or not tokens or source.length == 0:
            return
        n = min(len(tokens), source.length, self.max_tokens)
        if n <= 0:
            return
        key = tuple(tokens[:n])
        entry = self.manager.share(source, n)
        old = self._entries.pop(key, None)
        if old is not None:
            self.total_tokens -= len(key)
            self.manager.release(old)
        self._entries[key] = entry
        self.total_tokens += len(key)
        self._evict()

    def clear(self) -> None:
        for handle in self._entries.values():
            self.manager.release(handle)
        self._entries.clear()
        self.total_tokens = 0

    def __len__(self) -> int:
        return len(self._entries)

    def _evict(self) -> None:
        while self.total_tokens > self.max_tokens and self._entries:
            key, handle = self._entries.popitem(last=False)
            self.total_tokens -= len(key)
            self.manager.release(handle)


def _common_prefix(left: Sequence[int], right: Sequence[int], limit: int) -> int:
    n, top = 0, min(len(left), len(right), limit)
    while n < top and left[n] == right[n]:
        n += 1
    return n
