"""Planned prefill launches (longest items first, the heaviest cut in two and merged).

A planned launch must produce the rows of the default grid (within the bf16/f16
tolerance of 2e-2: a split item's halves are merged in f32 in another order) and of the
oracle; the same plan launched again (one per layer) gives identical rows and leaves the
split counters zero; a refused page in a split item is flagged and the next call is clean.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from hayate_b200 import PagedKVCacheManager, ops
from hayate_b200 import workloads as W

import oracle

pytestmark = pytest.mark.gpu


def build(lengths, query_len, dtype=torch.bfloat16, seed=0):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    pages = sum(math.ceil((n + query_len) / 128) for n in lengths) + 2
    m = PagedKVCacheManager(1, 8, 128, pages * 128, 128, len(lengths), dtype, "cuda")
    W.shuffle_free_pages(m, seed)
    hs = [m.allocate() for _ in lengths]
    for h, n in zip(hs, lengths):
        W.fill_history(m, h, n, gen)
    q, k, v = W.step_inputs(m, hs, query_len, 32, gen)
    batch = m.begin_batch(hs, query_len)
    batch.write_layer(0, k, v)
    return m, hs, batch, q


def oracle_rows(m, batch, q, requests=None):
    return oracle.paged_attention(q.float().cpu().numpy(), m.k_cache.float().cpu().numpy(),
                                  m.v_cache.float().cpu().numpy(), 0,
                                  batch.page_table.cpu().numpy().astype(np.int64),
                                  batch.cache_lens.cpu().numpy(), m.page_size, requests=requests)


CASES = [
    ([2998, 4045, 1590, 2020, 1436, 3762, 183, 2532], 512),   # config 3: the default grid
    ([1100, 516, 2089, 965, 4058, 3682, 3868, 3109], 512),    # longest first, no split
    ([0, 9000], 300),                                          # split items
    ([20000], 512),                                            # split items
    ([40], 40),
]
SPLIT = ([0, 9000], 300)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
@pytest.mark.parametrize("lengths, query_len", CASES, ids=str)
def test_planned_prefill_matches_default_grid_and_oracle(lengths, query_len, dtype):
    m, hs, batch, q = build(lengths, query_len, dtype, seed=len(lengths) + query_len)
    planned = batch.prefill_schedule(q)
    out = batch.attend_layer(q, 0)
    m.prefill_plan = False
    ref = m.begin_batch(hs, query_len).attend_layer(q, 0)
    torch.cuda.synchronize()
    m.check_device_errors()
    assert (out.float() - ref.float()).abs().max().item() <= 2e-2
    sample = list(range(min(2, len(lengths))))
    err = np.abs(out.float().cpu().numpy()[sample] - oracle_rows(m, batch, q, sample)[sample]).max()
    assert err <= 2e-2, err
    if planned is not None:  # a planned launch ran: its split counters are back at zero
        items, splits = planned
        assert items.shape[1] == 4
        if splits:
            ws = m.prefill_workspace(splits)
            assert int(ws[: 4 * splits].view(torch.int32).abs().sum().item()) == 0


def test_plan_choices():
    """Config 3 keeps the default grid, a U[0, 4096] batch it does not suit is reordered,
    and few long items are cut in two."""
    assert batch_plan(*CASES[0]) is None
    items, splits = batch_plan(*CASES[1])
    assert items.shape[0] == 8 * 4 * 16 and splits == 0
    items, splits = batch_plan(*SPLIT)
    assert splits > 0


def batch_plan(lengths, query_len):
    m, hs, batch, q = build(lengths, query_len, seed=1)
    return batch.prefill_schedule(q)


def test_split_plan_is_deterministic():
    lengths, query_len = SPLIT
    m, hs, batch, q = build(lengths, query_len, seed=3)
    planned = batch.prefill_schedule(q)
    assert planned is not None and planned[1] > 0  # this batch gets split items
    outs = [batch.attend_layer(q, 0) for _ in range(4)]  # one plan, several layers
    torch.cuda.synchronize()
    m.check_device_errors()
    assert all(torch.equal(outs[0], o) for o in outs[1:])


def test_planned_prefill_refused_page_then_clean_call():
    lengths, query_len = SPLIT
    m, hs, batch, q = build(lengths, query_len, seed=5)
    items, splits = batch.prefill_schedule(q)
    assert splits > 0
    table = batch.page_table.clone()
    table[1, 3] = m.num_pages + 1  # request 1 (prefix 9000): its items are the split ones
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = m.prefill_workspace(splits)
    ops.prefill_attention_planned(q, m.k_cache, m.v_cache, 0, table, batch.cache_lens_i32, 128, items,
                                  splits, workspace=ws, error_word=err)
    torch.cuda.synchronize()
    assert "page id outside the pool" in ops.read_device_errors(err)
    assert int(ws[: 4 * splits].view(torch.int32).abs().sum().item()) == 0  # counters reset
    out = batch.attend_layer(q, 0)
    torch.cuda.synchronize()
    m.check_device_errors()
    err2 = np.abs(out.float().cpu().numpy()[[1]] - oracle_rows(m, batch, q, [1])[[1]]).max()
    assert err2 <= 2e-2, err2


def test_planned_prefill_refused_request_both_halves_exit_early():
    """A request refused before any load (negative cache length): both halves of its cut
    items take the early path with empty partials; its rows are zeros, the counters end
    at zero and the next call is clean."""
    lengths, query_len = SPLIT
    m, hs, batch, q = build(lengths, query_len, seed=6)
    items, splits = batch.prefill_schedule(q)
    lens = batch.cache_lens_i32.clone()
    lens[1] = -1
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = m.prefill_workspace(splits)
    out = ops.prefill_attention_planned(q, m.k_cache, m.v_cache, 0, batch.page_table, lens, 128, items,
                                        splits, workspace=ws, error_word=err)
    torch.cuda.synchronize()
    assert "kv length needs more pages than the page table row holds" in ops.read_device_errors(err)
    assert float(out[1].float().abs().max()) == 0.0
    assert int(ws[: 4 * splits].view(torch.int32).abs().sum().item()) == 0
    good = batch.attend_layer(q, 0)
    torch.cuda.synchronize()
    m.check_device_errors()
    err2 = np.abs(good.float().cpu().numpy()[[1]] - oracle_rows(m, batch, q, [1])[[1]]).max()
    assert err2 <= 2e-2, err2
