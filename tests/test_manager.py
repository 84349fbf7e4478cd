"""Host-side page manager: the reference's own CPU tests plus sharing/copy-on-write.

Mirrors ``tests/test_paged_cache.py:10-51`` of hayate-exp (allocation, import,
snapshot, release, exhaustion) and checks that, given the same free-list order,
the manager builds exactly the page tables the reference built for the golden
cases.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_util import CASES, load_golden, make_inputs, shuffled_free_pages
from hayate_b200 import Cache, PagedKVCacheManager


def make_manager(max_cache_tokens=8, page_size=2, max_requests=2):
    return PagedKVCacheManager(num_layers=2, num_kv_heads=1, head_dim=4,
                               max_cache_tokens=max_cache_tokens, page_size=page_size,
                               max_requests=max_requests, dtype=torch.float32, device="cpu")


def test_import_snapshot_and_release_reuse_pages():
    manager = make_manager()
    values = torch.arange(24, dtype=torch.float32).reshape(2, 1, 3, 4)
    handle = manager.allocate_for_request(Cache.from_tensors(values, values + 1))
    original = list(handle.pages)
    snap = manager.snapshot(handle)
    assert handle.length == 3 and len(original) == 2
    torch.testing.assert_close(snap.k, values)
    torch.testing.assert_close(snap.v, values + 1)
    manager.release(handle)
    replacement = manager.allocate()
    manager.reserve(replacement, 3)
    assert set(replacement.pages) == set(original)


def test_pool_reports_exhausted_pages():
    manager = make_manager(max_cache_tokens=4)
    first, second = manager.allocate(), manager.allocate()
    manager.reserve(first, 4)
    with pytest.raises(MemoryError):
        manager.reserve(second, 1)


def test_slot_exhaustion_and_release_is_idempotent():
    manager = make_manager(max_requests=1)
    handle = manager.allocate()
    with pytest.raises(MemoryError):
        manager.allocate()
    manager.release(handle)
    manager.release(handle)
    assert manager.allocate().slot == 0


@pytest.mark.parametrize("call", ["reserve", "truncate", "snapshot", "begin_batch", "commit_batch", "share"])
def test_released_handle_is_rejected(call):
    manager = make_manager(page_size=128, max_cache_tokens=512)
    handle = manager.allocate()
    manager.release(handle)
    with pytest.raises(RuntimeError):
        {"reserve": lambda: manager.reserve(handle, 1),
         "truncate": lambda: manager.truncate(handle, 0),
         "snapshot": lambda: manager.snapshot(handle),
         "begin_batch": lambda: manager.begin_batch([handle], 1),
         "commit_batch": lambda: manager.commit_batch([handle], 1),
         "share": lambda: manager.share(handle, 0)}[call]()


def test_begin_batch_argument_errors():
    manager = make_manager(page_size=128, max_cache_tokens=512)
    handle = manager.allocate()
    with pytest.raises(ValueError):
        manager.begin_batch([], 1)
    with pytest.raises(ValueError):
        manager.begin_batch([handle], 0)
    with pytest.raises(ValueError):
        manager.begin_batch([handle, handle], 1)
    with pytest.raises(MemoryError):
        manager.begin_batch([handle], 513)
    small = make_manager(page_size=64, max_cache_tokens=512)
    with pytest.raises(ValueError):
        small.begin_batch([small.allocate()], 1)
    with pytest.raises(ValueError):
        PagedKVCacheManager(1, 1, 4, 16, 96, 1, torch.float32, "cpu")


def test_begin_batch_pool_full_has_no_side_effects():
    manager = make_manager(page_size=128, max_cache_tokens=256, max_requests=3)
    a, b = manager.allocate(), manager.allocate()
    manager.reserve(a, 200)
    with pytest.raises(MemoryError):
        manager.begin_batch([a, b], 100)  # a needs 1 more page (300 > 256 -> capacity) ...
    assert len(manager._free_pages) == 0 and len(b.pages) == 0


def test_commit_requires_reserved_space():
    manager = make_manager(page_size=128, max_cache_tokens=512)
    handle = manager.allocate()
    manager.begin_batch([handle], 5)
    manager.commit_batch([handle], 5)
    assert handle.length == 5
    with pytest.raises(RuntimeError):
        manager.commit_batch([handle], 200)


def test_begin_batch_metadata_layout():
    manager = make_manager(page_size=128, max_cache_tokens=1024, max_requests=3)
    a, b = manager.allocate(), manager.allocate()
    manager.reserve(a, 300)
    a.length = 300
    batch = manager.begin_batch([a, b], 2)
    assert batch.page_table.dtype == torch.int32 and batch.cache_lens.dtype == torch.int64
    assert batch.cache_lens.tolist() == [300, 0]
    assert batch.cache_lens_i32.tolist() == [300, 0]
    assert batch.page_table.tolist() == [[0, 1, 2], [3, -1, -1]]
    assert batch.max_kv_len == 302 and batch.page_size == 128


def test_share_refcounts_and_release_order():
    manager = make_manager(page_size=128, max_cache_tokens=1024, max_requests=4)
    src = manager.allocate()
    manager.reserve(src, 300)
    src.length = 300
    twin = manager.share(src, 256)
    assert twin.pages == src.pages[:2] and twin.length == 256
    assert [manager.page_refcount(p) for p in src.pages] == [2, 2, 1]
    free_before = len(manager._free_pages)
    manager.release(src)
    assert len(manager._free_pages) == free_before + 1  # only the unshared page came back
    assert [manager.page_refcount(p) for p in twin.pages] == [1, 1]
    manager.release(twin)
    assert len(manager._free_pages) == manager.num_pages
    with pytest.raises(ValueError):
        manager.share(manager.allocate(), 1)


def test_write_into_shared_page_copies_it_first():
    manager = PagedKVCacheManager(1, 1, 4, 1024, 128, 4, torch.float32, "cpu")
    values = torch.randn(1, 1, 200, 4)
    src = manager.allocate_for_request(Cache.from_tensors(values, -values))
    twin = manager.share(src, 150)  # shares both pages, the second one partially
    shared_second = twin.pages[1]
    manager.begin_batch([twin], 1)  # writes logical position 150: inside the shared page
    assert twin.pages[0] == src.pages[0]
    assert twin.pages[1] != shared_second and src.pages[1] == shared_second
    assert manager.page_refcount(shared_second) == 1
    # the copy carries the shared prefix of that page
    torch.testing.assert_close(manager.snapshot(twin, 150).k, values[:, :, :150])
    torch.testing.assert_close(manager.snapshot(src).v, -values)


def test_truncate_returns_pages():
    manager = make_manager(page_size=128, max_cache_tokens=1024)
    handle = manager.allocate()
    manager.reserve(handle, 512)
    handle.length = 512
    manager.truncate(handle, 129)
    assert len(handle.pages) == 2 and len(manager._free_pages) == 6
    with pytest.raises(ValueError):
        manager.truncate(handle, 130)


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_page_tables_match_reference(case):
    """Same free-list order in, same page tables out as the reference's begin_batch."""
    golden = load_golden(case.name)
    inputs = make_inputs(case)
    manager = PagedKVCacheManager(case.num_layers, case.num_kv_heads, case.head_dim,
                                  case.max_cache_tokens, case.page_size, case.batch,
                                  torch.float32, "cpu")
    manager._free_pages = shuffled_free_pages(manager.num_pages, case.seed)
    handles = []
    for hk, hv in zip(inputs["hist_k"], inputs["hist_v"]):
        cache = Cache.from_tensors(torch.from_numpy(hk), torch.from_numpy(hv)) if hk.shape[2] else None
        handles.append(manager.allocate_for_request(cache))
    batch = manager.begin_batch(handles, case.query_len)
    table = batch.page_table.numpy()
    ref = golden["page_table"]
    np.testing.assert_array_equal(golden["handle_pages"], [len(h.pages) for h in handles])
    for row, count in enumerate(golden["handle_pages"]):
        np.testing.assert_array_equal(table[row, :count], ref[row, :count])
    np.testing.assert_array_equal(batch.cache_lens.numpy(), golden["cache_lens"])


def test_kernels_refuse_cpu_tensors():
    manager = make_manager(page_size=128, max_cache_tokens=512)
    handle = manager.allocate()
    batch = manager.begin_batch([handle], 1)
    with pytest.raises(RuntimeError, match="CUDA"):
        batch.write_layer(0, torch.zeros(1, 1, 1, 4), torch.zeros(1, 1, 1, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        batch.attend_layer(torch.zeros(1, 1, 1, 4), 0)


def test_persistent_page_table_tracks_every_page_change():
    """The slot-indexed rows behind each step's page table follow every mutation."""
    manager = PagedKVCacheManager(1, 1, 4, 64 * 128, 128, 6, torch.float32, "cpu")
    values = torch.randn(1, 1, 300, 4)
    a = manager.allocate_for_request(Cache.from_tensors(values, values))
    b = manager.share(a, 200)                 # aliases a's first two pages
    c = manager.allocate()
    manager.reserve(c, 1000)                  # 8 pages, wider than the initial rows
    c.length = 900
    manager.truncate(c, 300)                  # drop pages 3..7
    manager.release(manager.share(a, 256))    # a slot that comes and goes
    d = manager.allocate()                    # reuses the released slot
    handles = [a, b, c, d]
    for step in range(3):
        batch = manager.begin_batch(handles, 130)   # b's write lands in a shared page: COW
        width = batch.page_table.shape[1]
        for row, h in enumerate(handles):
            expected = (h.pages + [-1] * width)[:width]
            assert batch.page_table[row].tolist() == expected, (step, row)
        manager.commit_batch(handles, 130)
    assert manager.page_refcount(b.pages[1]) == 1 and b.pages[0] == a.pages[0]


def test_packed_batch_layout_and_commit():
    """One query length per request: a packed batch on one token axis."""
    manager = make_manager(page_size=128, max_cache_tokens=4096, max_requests=4)
    a, b, c = manager.allocate(), manager.allocate(), manager.allocate()
    manager.reserve(a, 300)
    a.length = 300
    batch = manager.begin_batch([a, b, c], [1, 130, 5])
    lay = batch.layout
    assert lay.query_lens == [1, 130, 5] and lay.total_tokens == 136
    assert lay.q_start.tolist() == [0, 1, 131] and lay.q_len.tolist() == [1, 130, 5]
    assert lay.decode_ids.tolist() == [0] and lay.prefill_ids.tolist() == [1, 2]
    assert lay.token_request.tolist() == [0] + [1] * 130 + [2] * 5
    assert batch.cache_lens.tolist() == [300, 0, 0] and batch.query_len == 130
    assert batch.max_kv_len == 301
    assert [len(h.pages) for h in (a, b, c)] == [3, 2, 1]
    manager.commit_batch([a, b, c], [1, 130, 5])
    assert [h.length for h in (a, b, c)] == [301, 130, 5]
    # a uniform batch after it has no packed layout
    assert manager.begin_batch([a, b], 2).layout is None


def test_packed_batch_argument_errors():
    manager = make_manager(page_size=128, max_cache_tokens=1024, max_requests=3)
    a, b = manager.allocate(), manager.allocate()
    with pytest.raises(ValueError):
        manager.begin_batch([a, b], [1])
    with pytest.raises(ValueError):
        manager.begin_batch([a, b], [1, 0])
    with pytest.raises(ValueError):
        manager.commit_batch([a, b], [1, 2, 3])
    with pytest.raises(MemoryError):
        manager.begin_batch([a, b], [1, 2000])


def test_copy_on_write_follows_sharing_only():
    """Requests that never shared pages skip the copy-on-write check; shared ones get it."""
    manager = PagedKVCacheManager(1, 1, 4, 2048, 128, 6, torch.float32, "cpu")
    values = torch.randn(1, 1, 200, 4)
    a = manager.allocate_for_request(Cache.from_tensors(values, values))
    plain = manager.allocate_for_request(Cache.from_tensors(values, values))
    assert not a.aliased and not plain.aliased
    twin = manager.share(a, 150)
    assert a.aliased and twin.aliased and not plain.aliased
    empty = manager.share(plain, 0)           # nothing aliased: flags unchanged
    assert not plain.aliased and not empty.aliased
    shared_page = twin.pages[1]
    manager.begin_batch([a, twin, plain], [1, 1, 1])
    # both append into the shared second page: the first to write (a) gets a copy
    assert a.pages[1] != shared_page and twin.pages[1] == shared_page
    assert manager.page_refcount(a.pages[1]) == 1 and manager.page_refcount(shared_page) == 1
    assert a.pages[0] == twin.pages[0] and manager.page_refcount(a.pages[0]) == 2
    manager.release(twin)
    assert not twin.aliased


def test_copy_on_write_pages_counted_before_any_change():
    """A step whose growth fits but whose copy-on-write pages do not fails up front: no
    handle gains a page and no reference count moves."""
    manager = PagedKVCacheManager(1, 1, 4, 6 * 128, 128, 6, torch.float32, "cpu")
    values = torch.randn(1, 1, 200, 4)
    src = manager.allocate_for_request(Cache.from_tensors(values, values))   # pages 0, 1
    twins = [manager.share(src, 200) for _ in range(3)]                      # page 1 held by 4
    grow = manager.allocate_for_request(Cache.from_tensors(values[:, :, :128], values[:, :, :128]))
    assert len(manager._free_pages) == 3
    # grow needs 1 new page; the 3 twins each append into page 1 (4 holders): 3 copies
    handles = [grow] + twins
    before = ([list(h.pages) for h in handles], manager._page_refs.copy(), list(manager._free_pages))
    with pytest.raises(MemoryError):
        manager.begin_batch(handles, 1)
    assert [list(h.pages) for h in handles] == before[0]
    assert np.array_equal(manager._page_refs, before[1]) and manager._free_pages == before[2]
    # without the growing request the three copies fit exactly, and the last writer keeps
    # nothing shared: src still holds the original page alone
    manager.begin_batch(twins, 1)
    assert len(manager._free_pages) == 0
    assert manager.page_refcount(src.pages[1]) == 1
    assert len({t.pages[1] for t in twins} | {src.pages[1]}) == 4


def test_copy_on_write_count_is_exact_when_all_holders_write():
    """Every holder of a page writing into it needs one copy fewer than holders."""
    manager = PagedKVCacheManager(1, 1, 4, 4 * 128, 128, 4, torch.float32, "cpu")
    values = torch.randn(1, 1, 200, 4)
    src = manager.allocate_for_request(Cache.from_tensors(values, values))   # pages 0, 1
    twin = manager.share(src, 200)
    assert len(manager._free_pages) == 2
    manager.begin_batch([src, twin], 1)  # page 1 has 2 holders, both write: 1 copy
    assert len(manager._free_pages) == 1 and src.pages[1] != twin.pages[1]


def test_shared_workspaces_zero_counters_a_new_layout_reaches():
    """A grow-only workspace shared by layouts of different sizes: bytes a smaller layout
    used for partials must be zero again before a larger layout uses them as counters."""
    from hayate_b200 import ops

    m = PagedKVCacheManager(1, 8, 128, 64 * 128, 128, 128, torch.bfloat16, "cpu")
    m.split_tokens = 1024
    big = m.workspace_for(100, 1, 32, 4096)  # allocates for 100 requests
    big.fill_(0xFF)  # partials of the big layout (counters of a finished launch are zero...)
    big[: ops.attention_counter_bytes(100, 8)] = 0  # ... as the kernels leave them
    small = m.workspace_for(10, 1, 32, 4096)
    assert small.data_ptr() == big.data_ptr()
    small[ops.attention_counter_bytes(10, 8):] = 0xAB  # the small layout's partials
    mid = m.workspace_for(60, 1, 32, 4096)
    assert mid.data_ptr() == big.data_ptr()
    assert int(mid[: ops.attention_counter_bytes(60, 8)].abs().sum()) == 0

    pw = m.prefill_workspace(100)
    pw.fill_(0xFF)
    pw[: ops.prefill_counter_bytes(100)] = 0
    pw2 = m.prefill_workspace(10)
    pw2[ops.prefill_counter_bytes(10):] = 0xAB
    pw3 = m.prefill_workspace(80)
    assert pw3.data_ptr() == pw.data_ptr()
    assert int(pw3[: ops.prefill_counter_bytes(80)].abs().sum()) == 0
