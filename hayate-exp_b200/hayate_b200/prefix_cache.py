"""Prefix cache whose entries alias physical KV pages instead of holding copies.

It offers the calls hayate's ``PrefixCache`` offers (``hayate/engine/prefix_cache.py:18-100``):
``get(tokens, max_prefix_len)`` finds the longest stored prefix of a prompt, ``put(tokens,
source)`` stores one under a token budget with least-recently-used eviction, ``clear()``
empties it. What an entry is differs. hayate clones a contiguous K/V snapshot on ``put``
and copies it back into fresh pages on a hit (``hayate/engine/paged_cache.py:153-190``).
Here an entry is a handle made by ``PagedKVCacheManager.share``: it holds references on
the source's pages, so ``put`` and a hit move no K/V bytes, and a hit's pages stay shared
until the new request writes into one of them (copy-on-write in ``begin_batch``).
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass
from itertools import takewhile
from typing import Sequence

from .paged_cache import PagedCacheHandle, PagedKVCacheManager


@dataclass(frozen=True)
class PrefixCacheMatch:
    """How many leading tokens were found, and a new handle aliasing their pages."""

    length: int
    handle: PagedCacheHandle | None


_MISS = PrefixCacheMatch(0, None)


def _shared_prefix_len(a: Sequence[int], b: Sequence[int], cap: int) -> int:
    """Number of equal leading tokens of ``a`` and ``b``, at most ``cap``."""
    return sum(1 for _ in takewhile(lambda pair: pair[0] == pair[1], zip(a[:cap], b[:cap])))


class PagedPrefixCache:
    """Token-prefix -> page-aliasing handle map of one manager, evicted oldest-use first.

    Every entry owns its handle: eviction, replacement and ``clear`` release it, which
    drops the entry's references on the pages (a page is freed once no request or entry
    references it).
    """

    def __init__(self, manager: PagedKVCacheManager, max_tokens: int):
        if max_tokens < 0:
            raise ValueError(f"max_tokens is a token budget and cannot be negative (got {max_tokens})")
        self.manager = manager
        self.max_tokens = max_tokens
        self.total_tokens = 0
        # least recently used first; a hit or a store moves the entry to the end
        self._entries: OrderedDict[tuple[int, ...], PagedCacheHandle] = OrderedDict()

    def get(self, tokens: Sequence[int], max_prefix_len: int | None = None) -> PrefixCacheMatch:
        """The longest stored prefix of ``tokens`` (at most ``max_prefix_len`` long).

        On a hit the match carries a NEW handle sharing that prefix's pages; the caller owns
        it and releases it like any request handle. Ties keep the first entry found.
        """
        if not tokens or not self._entries or self.max_tokens == 0:
            return _MISS
        prompt = tuple(tokens)
        cap = len(prompt) if max_prefix_len is None else min(len(prompt), max_prefix_len)
        if cap < 1:
            return _MISS
        hit_key, hit_len = None, 0
        for key, entry in self._entries.items():
            # an entry can only serve as many tokens as its handle still holds
            n = _shared_prefix_len(prompt, key, min(cap, entry.length))
            if n > hit_len:
                hit_key, hit_len = key, n
                if n == cap:  # nothing can beat a full-length match
                    break
        if hit_key is None:
            return _MISS
        self._entries.move_to_end(hit_key)
        return PrefixCacheMatch(hit_len, self.manager.share(self._entries[hit_key], hit_len))

    def put(self, tokens: Sequence[int], source: PagedCacheHandle) -> None:
        """Store the longest prefix of ``tokens`` that ``source`` holds and the budget allows,
        as an alias of ``source``'s pages (no copy). A key stored before is replaced."""
        n = min(len(tokens), source.length, self.max_tokens) if tokens else 0
        if n < 1:
            return
        key = tuple(tokens[:n])
        alias = self.manager.share(source, n)
        replaced = self._entries.pop(key, None)
        if replaced is not None:
            self._drop(key, replaced)
        self._entries[key] = alias
        self.total_tokens += n
        while self.total_tokens > self.max_tokens and self._entries:
            self._drop(*self._entries.popitem(last=False))

    def clear(self) -> None:
        """Release every entry's handle and forget all prefixes."""
        while self._entries:
            self._drop(*self._entries.popitem())

    def __len__(self) -> int:
        return len(self._entries)

    def _drop(self, key: tuple[int, ...], handle: PagedCacheHandle) -> None:
        self.total_tokens -= len(key)
        self.manager.release(handle)
