"""Page-sharing prefix cache: the reference PrefixCache's LRU behaviour, no K/V copies.

Follows hayate-exp's ``tests/test_cache.py`` (prefix lookups, immutability of stored
entries) on the host, with pools on the CPU.
"""

from __future__ import annotations

import pytest
import torch

from hayate_b200 import Cache, PagedKVCacheManager, PagedPrefixCache


def make(max_tokens=4096, pages=64):
    manager = PagedKVCacheManager(1, 1, 4, pages * 128, 128, 16, torch.float32, "cpu")
    return manager, PagedPrefixCache(manager, max_tokens)


def request(manager, tokens):
    values = torch.arange(len(tokens) * 4, dtype=torch.float32).reshape(1, 1, len(tokens), 4)
    return manager.allocate_for_request(Cache.from_tensors(values, -values))


def test_put_and_get_share_pages_without_copying():
    manager, cache = make()
    tokens = list(range(300))
    src = request(manager, tokens)
    free_before = len(manager._free_pages)
    cache.put(tokens, src)
    assert len(manager._free_pages) == free_before  # no new pages for the entry
    match = cache.get(tokens + [7, 8], max_prefix_len=301)
    assert match.length == 300
    assert match.handle.pages == src.pages and match.handle.length == 300
    assert all(manager.page_refcount(p) == 3 for p in src.pages)  # request + entry + hit
    torch.testing.assert_close(manager.snapshot(match.handle).k, manager.snapshot(src).k)


def test_longest_prefix_and_limits():
    manager, cache = make()
    a, b = list(range(10)), list(range(5)) + [99] * 20
    cache.put(a, request(manager, a))
    cache.put(b, request(manager, b))
    assert cache.get(list(range(8))).length == 8
    assert cache.get(list(range(5)) + [99, 99]).length == 7
    assert cache.get(list(range(10)), max_prefix_len=3).length == 3
    assert cache.get([42]).length == 0 and cache.get([42]).handle is None
    assert cache.get([]).length == 0


def test_entries_survive_source_release_and_truncate():
    manager, cache = make()
    tokens = list(range(200))
    src = request(manager, tokens)
    expected = manager.snapshot(src).k.clone()
    cache.put(tokens, src)
    manager.truncate(src, 10)
    manager.release(src)
    hit = cache.get(tokens)
    torch.testing.assert_close(manager.snapshot(hit.handle).k, expected)


def test_hit_appends_copy_on_write_and_keep_entry_intact():
    manager, cache = make()
    tokens = list(range(150))
    src = request(manager, tokens)
    cache.put(tokens, src)
    manager.release(src)
    hit = cache.get(tokens + [1], max_prefix_len=149)  # shares a partial second page
    assert hit.length == 149
    before = [manager.page_refcount(p) for p in hit.handle.pages]
    manager.begin_batch([hit.handle], 1)  # writes position 149 inside the shared page
    assert before[1] == 2 and manager.page_refcount(hit.handle.pages[1]) == 1
    again = cache.get(tokens)
    assert again.length == 150


def test_lru_eviction_releases_pages():
    manager, cache = make(max_tokens=300)
    first, second = list(range(200)), list(range(1000, 1200))
    h1, h2 = request(manager, first), request(manager, second)
    cache.put(first, h1)
    manager.release(h1)
    cache.put(second, h2)  # over budget: the least recently used entry goes
    manager.release(h2)
    assert len(cache) == 1 and cache.total_tokens == 200
    assert cache.get(first).length == 0
    free = len(manager._free_pages)
    cache.clear()
    assert len(manager._free_pages) == free + 2 and cache.total_tokens == 0


def test_zero_budget_and_validation():
    manager, cache = make(max_tokens=0)
    h = request(manager, [1, 2, 3])
    cache.put([1, 2, 3], h)
    assert len(cache) == 0 and cache.get([1, 2, 3]).length == 0
    with pytest.raises(ValueError):
        PagedPrefixCache(manager, -1)
