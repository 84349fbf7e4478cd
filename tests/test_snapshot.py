"""KVSnapshot, the exchange type of ``snapshot``/``import_cache`` (CPU)."""

from __future__ import annotations

import os
import sys

import pytest
import torch

from hayate_b200 import Cache, KVSnapshot, PagedKVCacheManager

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def _kv(tokens=10, layers=2, heads=3, dim=4):
    k = torch.arange(layers * heads * tokens * dim, dtype=torch.float32).view(layers, heads, tokens, dim)
    return k, -k


def test_views_and_clones():
    k, v = _kv()
    snap = KVSnapshot.from_tensors(k, v)
    assert snap.length == snap.capacity == 10
    view = snap.slice(4)
    assert view.length == 4 and view.k.data_ptr() == k.data_ptr()  # a view: no copy
    kept = snap.slice(4, clone=True)
    assert kept.k.is_contiguous() and kept.k.data_ptr() != k.data_ptr()
    k.add_(1000)  # later writes to the source reach the view, not the clone
    assert torch.equal(view.k, k[:, :, :4])
    assert torch.equal(kept.k, k[:, :, :4] - 1000)
    assert snap.slice(0).length == 0
    assert KVSnapshot().slice(0).length == 0


def test_refusals():
    k, v = _kv()
    with pytest.raises(ValueError):
        KVSnapshot(k, v[:, :, :3])
    with pytest.raises(ValueError):
        KVSnapshot(k, None)
    with pytest.raises(ValueError):
        KVSnapshot(k[0], v[0])
    with pytest.raises(ValueError):
        KVSnapshot(k, v).slice(11)
    with pytest.raises(ValueError):
        KVSnapshot(k, v).slice(-1)


def test_extended_is_a_new_snapshot():
    k, v = _kv(tokens=6)
    a = KVSnapshot(k, v)
    b = a.extended(k[:, :, :2], v[:, :, :2])
    assert a.length == 6 and b.length == 8
    assert torch.equal(b.k[:, :, 6:], k[:, :, :2]) and torch.equal(b.v[:, :, :6], v)
    assert KVSnapshot().extended(k, v).length == 6
    assert Cache is KVSnapshot


def test_round_trip_through_the_manager():
    m = PagedKVCacheManager(2, 3, 4, 8 * 128, 128, 2, torch.float32, "cpu")
    k, v = _kv(tokens=300)
    h = m.allocate_for_request(KVSnapshot(k, v))
    snap = m.snapshot(h)
    assert isinstance(snap, KVSnapshot) and snap.length == 300
    assert torch.equal(snap.k, k) and torch.equal(snap.v, v)
    h2 = m.allocate_for_request(snap.slice(129))
    assert torch.equal(m.snapshot(h2).k, k[:, :, :129])


def test_reference_prefix_cache_accepts_snapshots():
    """hayate's own PrefixCache stores a snapshot (slice with clone) and serves a hit (slice)."""
    if not os.path.isdir(os.path.join(REF_DIR, "hayate")):
        pytest.skip("reference not installed in baseline/_ref")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    from hayate.engine.prefix_cache import PrefixCache

    m = PagedKVCacheManager(2, 3, 4, 8 * 128, 128, 3, torch.float32, "cpu")
    k, v = _kv(tokens=200)
    h = m.allocate_for_request(KVSnapshot(k, v))
    cache = PrefixCache(max_tokens=1000)
    tokens = list(range(200))
    cache.put(tokens, m.snapshot(h))
    m.release(h)
    match = cache.get(tokens[:150] + [-1, -2])
    assert match.length == 150
    h2 = m.allocate_for_request(match.cache)
    assert h2.length == 150 and torch.equal(m.snapshot(h2).k, k[:, :, :150])
