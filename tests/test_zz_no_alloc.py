"""The allocation-free decode entry point against the workspace one, through the C ABI.

``hyt_decode_attention_noalloc`` serves callers that cannot allocate device
memory (a C/FFI host that only borrows another framework's tensors, or a
serving loop that must not call cudaMalloc while running): its split scratch is
a static device array inside the library. This file is collected last so that
a failure here never hides the other tests; it also passes alone.
"""

from __future__ import annotations

import math

import pytest
import torch

from hayate_b200 import PagedKVCacheManager, _lib, ops
from hayate_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = 2e-2  # bf16 attention tolerance used by every GPU parity test


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


def _args(manager, batch, q, out):
    L, _, H, cap, D = manager.k_cache.shape
    return [q.data_ptr(), _lib.int64_array(q.stride()[:3]), manager.k_cache.data_ptr(),
            manager.v_cache.data_ptr(), L, 0, cap, batch.page_table.data_ptr(),
            batch.page_table.stride(0), batch.cache_lens_i32.data_ptr(), out.data_ptr(),
            _lib.int64_array(out.stride()[:3]), q.shape[0], 1, 32, H, D, 128,
            _lib.HYT_DTYPE_BF16, 1.0 / math.sqrt(D), batch.max_kv_len]


def test_noalloc_decode_matches_workspace_decode_on_two_calls():
    lengths = [5000, 130, 6143, 2048, 1, 4097]
    manager, batch, q = _decode_step(lengths, seed=17)
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    split = 512  # several splits per request, so the scratch carries partials and counters
    ws_bytes = ops.attention_workspace_bytes(len(lengths), 1, 32, 8, 128, batch.max_kv_len,
                                             torch.bfloat16, split)
    assert 0 < ws_bytes <= _lib.lib().hyt_attention_workspace_bytes(
        len(lengths), 1, 32, 8, 128, batch.max_kv_len, split, 0)
    workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    expected = torch.empty_like(q)
    rc = lib.hyt_decode_attention(*_args(manager, batch, q, expected), split, workspace.data_ptr(),
                                  ws_bytes, None, stream)
    _lib.check(rc, "hyt_decode_attention")
    for _ in range(2):  # the static scratch keeps the previous call's bytes
        got = torch.full_like(q, float("nan"))
        rc = lib.hyt_decode_attention_noalloc(*_args(manager, batch, q, got), split, None, stream)
        _lib.check(rc, "hyt_decode_attention_noalloc")
        torch.cuda.synchronize()
        err = (got.float() - expected.float()).abs().max().item()
        assert err <= TOL, err


def test_noalloc_decode_refuses_sizes_beyond_its_scratch():
    lengths = [8191] * 64
    manager, batch, q = _decode_step(lengths, seed=3)
    out = torch.empty_like(q)
    lib = _lib.lib()
    split = 64  # 128 splits x 64 requests x 8 heads: far beyond the static buffer
    need = lib.hyt_attention_workspace_bytes(64, 1, 32, 8, 128, batch.max_kv_len, split, 0)
    assert need > (8 << 20)
    rc = lib.hyt_decode_attention_noalloc(*_args(manager, batch, q, out), split, None,
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == -4
    assert "exceeds the static" in lib.hyt_last_error().decode()
