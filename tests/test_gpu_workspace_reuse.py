"""One manager's grow-only workspaces shared by launches of different sizes (GPU).

A serving loop reuses one decode workspace and one prefill-plan workspace for every step
while its batch sizes and schedules change. The counters at the start of a workspace must
be zero when a launch starts; a layout with more counters than an earlier, smaller one
covers bytes that the smaller one used for partials. These tests run large, then small,
then mid-size launches over the same buffers and check every launch's rows.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from hayate_b200 import PagedKVCacheManager, ops
from hayate_b200 import workloads as W

from test_gpu_parity import oracle_request_rows

pytestmark = pytest.mark.gpu

TOL = 2e-2  # bf16 attention tolerance of every GPU parity test


def _decode_phase(m, n_requests, kv_len, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    handles = [m.allocate() for _ in range(n_requests)]
    for h in handles:
        W.fill_history(m, h, kv_len - 1, gen)
    q, k, v = W.step_inputs(m, handles, 1, 32, gen)
    batch = m.begin_batch(handles, 1)
    out = batch.write_attend_layer(0, k, v, q)
    torch.cuda.synchronize()
    m.check_device_errors()
    return handles, batch, q, out


def test_decode_workspace_shared_by_batches_of_different_sizes():
    kv = 4000
    pages = 64 * math.ceil((kv + 1) / 128) + 8
    m = PagedKVCacheManager(1, 8, 128, pages * 128, 128, 128, torch.bfloat16, "cuda")
    m.split_tokens = 1024  # four splits a request: every launch uses the workspace
    W.shuffle_free_pages(m, 5)
    for n_requests, seed in ((64, 1), (8, 2), (40, 3)):  # large, small, then mid-size
        handles, batch, q, out = _decode_phase(m, n_requests, kv, seed)
        check = sorted({0, n_requests // 2, n_requests - 1, max(0, n_requests - 9)})
        ref = oracle_request_rows(m, batch, q, check)
        got = out.float().cpu().numpy()
        for b in check:
            err = float(np.abs(got[b] - ref[b]).max())
            assert err <= TOL, (n_requests, b, err)
        for h in handles:
            m.release(h)


def _cut_plan(lengths, query_len, n_cut):
    """Items in the default grid's order (request, head pair, query tile from the last), the
    first n_cut items with two or more key tiles cut in two at half their key tiles."""
    items, slot = [], 0
    tiles_q = -(-query_len // 128)
    for z, n in enumerate(lengths):
        for pair in range(16):
            for qt in reversed(range(tiles_q)):
                kt = (n + min(qt * 128 + 128, query_len) - 1) // 128 + 1
                tp = qt | (pair << 16)
                if slot < n_cut and kt >= 2:
                    h = kt // 2
                    items += [(z, tp, h << 16, 2 * slot), (z, tp, h | (0xFFFF << 16), 2 * slot + 1)]
                    slot += 1
                else:
                    items.append((z, tp, 0xFFFF << 16, -1))
    a = (np.array(items, dtype=np.int64) & 0xFFFFFFFF).astype(np.uint32).view(np.int32).reshape(-1, 4)
    return torch.from_numpy(a.copy()).cuda(), slot


def test_prefill_plan_workspace_shared_by_plans_of_different_sizes():
    """Plans with 128, then 8, then 96 split slots over one prefill workspace (the counters
    of 96 slots reach bytes the 8-slot plan used for partials); every launch against the
    same batch on the default grid."""
    lengths, T = [9000, 300, 6000, 2500], 300
    gen = torch.Generator(device="cuda").manual_seed(7)
    pages = sum(math.ceil((n + T) / 128) for n in lengths) + 2
    m = PagedKVCacheManager(1, 8, 128, pages * 128, 128, len(lengths), torch.bfloat16, "cuda")
    W.shuffle_free_pages(m, 7)
    hs = [m.allocate() for _ in lengths]
    for h, n in zip(hs, lengths):
        W.fill_history(m, h, n, gen)
    q, k, v = W.step_inputs(m, hs, T, 32, gen)
    batch = m.begin_batch(hs, T)
    batch.write_layer(0, k, v)
    ref = ops.prefill_attention_planned(q, m.k_cache, m.v_cache, 0, batch.page_table,
                                        batch.cache_lens_i32, 128, None, 0)
    for n_cut in (128, 8, 96):
        items, splits = _cut_plan(lengths, T, n_cut)
        assert splits == n_cut
        out = ops.prefill_attention_planned(q, m.k_cache, m.v_cache, 0, batch.page_table,
                                            batch.cache_lens_i32, 128, items, splits,
                                            workspace=m.prefill_workspace(splits),
                                            error_word=m.error_word)
        torch.cuda.synchronize()
        m.check_device_errors()
        err = float((out.float() - ref.float()).abs().max())
        assert err <= TOL, (n_cut, err)
