"""The allocation-free decode entry point against the workspace one, through the C ABI.

``hyt_decode_attention_noalloc`` serves callers that cannot allocate device
memory (a C/FFI host that only borrows another framework's tensors, or a
serving loop that must not call cudaMalloc while running): its split scratch is
a static device array inside the library that every call reuses. Both entry
points run the same kernel, so with the same ``split_tokens`` their outputs must
be bit-identical; anything else means a partial or counter left over in the
shared array leaked into a later call. This file is collected last so that a
failure here never hides the other tests; it also passes alone.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from hayate_b200 import PagedKVCacheManager, _lib, ops
from hayate_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = 2e-2  # bf16 attention tolerance of every GPU parity test (oracle comparison)
LENGTHS = [5000, 130, 6143, 2048, 1, 4097]


def _decode_step(lengths, seed=0):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    pages = sum(math.ceil((n + 1) / 128) for n in lengths) + 2
    manager = PagedKVCacheManager(1, 8, 128, pages * 128, 128, len(lengths), torch.bfloat16, "cuda")
    W.shuffle_free_pages(manager, seed)
    handles = [manager.allocate() for _ in lengths]
    for h, n in zip(handles, lengths):
        W.fill_history(manager, h, n, gen)
    q, k, v = W.step_inputs(manager, handles, 1, 32, gen)
    batch = manager.begin_batch(handles, 1)
    batch.write_layer(0, k, v)
    return manager, batch, q


def _args(manager, batch, q, out, table=None):
    L, _, H, cap, D = manager.k_cache.shape
    table = batch.page_table if table is None else table
    return [q.data_ptr(), _lib.int64_array(q.stride()[:3]), manager.k_cache.data_ptr(),
            manager.v_cache.data_ptr(), L, 0, cap, table.data_ptr(),
            table.stride(0), batch.cache_lens_i32.data_ptr(), out.data_ptr(),
            _lib.int64_array(out.stride()[:3]), q.shape[0], 1, 32, H, D, 128,
            _lib.HYT_DTYPE_BF16, 1.0 / math.sqrt(D), batch.max_kv_len]


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _with_workspace(manager, batch, q, split):
    """The existing entry point (caller-allocated workspace) with the same split size."""
    lib = _lib.lib()
    n = len(batch.cache_lens_i32)
    ws_bytes = ops.attention_workspace_bytes(n, 1, 32, 8, 128, batch.max_kv_len, torch.bfloat16, split)
    assert 0 < ws_bytes == lib.hyt_attention_workspace_bytes(n, 1, 32, 8, 128, batch.max_kv_len, split, 0)
    workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.full_like(q, float("nan"))
    _lib.check(lib.hyt_decode_attention(*_args(manager, batch, q, out), split, workspace.data_ptr(),
                                        ws_bytes, None, _stream()), "hyt_decode_attention")
    return out


def _noalloc(manager, batch, q, split, table=None, error_word=None):
    out = torch.full_like(q, float("nan"))
    err_ptr = None if error_word is None else error_word.data_ptr()
    rc = _lib.lib().hyt_decode_attention_noalloc(*_args(manager, batch, q, out, table), split,
                                                 err_ptr, _stream())
    _lib.check(rc, "hyt_decode_attention_noalloc")
    return out


def test_noalloc_decode_matches_workspace_decode_on_two_calls():
    manager, batch, q = _decode_step(LENGTHS, seed=17)
    split = 512  # several splits per request, so the scratch carries partials and counters
    expected = _with_workspace(manager, batch, q, split)
    for _ in range(2):  # the static scratch keeps the previous call's bytes
        got = _noalloc(manager, batch, q, split)
        torch.cuda.synchronize()
        assert torch.equal(got, expected)
    manager.check_device_errors()
    # and the rows are the attention the oracle computes on the same pool
    ref = oracle.paged_attention(q.float().cpu().numpy(), manager.k_cache.float().cpu().numpy(),
                                 manager.v_cache.float().cpu().numpy(), 0,
                                 batch.page_table.cpu().numpy().astype(np.int64),
                                 batch.cache_lens.cpu().numpy(), 128)
    err = float(np.abs(got.float().cpu().numpy() - ref).max())
    assert err <= TOL, err


def test_noalloc_library_split_matches_workspace_decode():
    """split_tokens 0: the library's own split size for this batch, on both entry points."""
    manager, batch, q = _decode_step(LENGTHS, seed=19)
    expected = _with_workspace(manager, batch, q, 0)
    for _ in range(2):
        got = _noalloc(manager, batch, q, 0)
        torch.cuda.synchronize()
        assert torch.equal(got, expected)
    manager.check_device_errors()


def test_noalloc_many_splits_then_few():
    """A call with many splits fills much of the array; a later call with fewer splits lays
    its partials out differently over the same bytes and must not read the old ones."""
    manager, batch, q = _decode_step(LENGTHS, seed=23)
    for split in (128, 2048, 256, 1024):
        got = _noalloc(manager, batch, q, split)
        expected = _with_workspace(manager, batch, q, split)
        torch.cuda.synchronize()
        assert torch.equal(got, expected), split
    manager.check_device_errors()


def test_noalloc_clean_call_after_a_refused_one():
    """A call the kernel refuses on the device (a page id outside the pool, planted in a copy
    of the page table: the error word gets the page-range bit and that split loads nothing)
    leaves the shared array in a state the next clean call must not inherit."""
    manager, batch, q = _decode_step(LENGTHS, seed=29)
    split = 512
    bad_table = batch.page_table.clone()
    bad_table[0, 3] = manager.num_pages + 5  # request 0 (5000 keys): its 512-key split 0 reads page 3
    error_word = torch.zeros(1, dtype=torch.int32, device="cuda")
    _noalloc(manager, batch, q, split, table=bad_table, error_word=error_word)
    torch.cuda.synchronize()
    problems = ops.read_device_errors(error_word)
    assert problems and any("page" in p for p in problems), problems
    got = _noalloc(manager, batch, q, split)
    expected = _with_workspace(manager, batch, q, split)
    torch.cuda.synchronize()
    assert torch.equal(got, expected)
    manager.check_device_errors()


def test_noalloc_decode_refuses_sizes_beyond_its_scratch():
    lengths = [8191] * 64
    manager, batch, q = _decode_step(lengths, seed=3)
    out = torch.empty_like(q)
    lib = _lib.lib()
    split = 64  # 128 splits x 64 requests x 8 heads: far beyond the static buffer
    need = lib.hyt_attention_workspace_bytes(64, 1, 32, 8, 128, batch.max_kv_len, split, 0)
    assert need > _lib.HYT_NOALLOC_SCRATCH_BYTES
    rc = lib.hyt_decode_attention_noalloc(*_args(manager, batch, q, out), split, None, _stream())
    assert rc == _lib.HYT_ERR_WORKSPACE
    assert "exceeds the static" in lib.hyt_last_error().decode()
