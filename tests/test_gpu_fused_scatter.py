"""write_attend_layer: the decode kernel writing the step's K/V rows itself.

``PagedKVBatch.write_attend_layer`` (``hyt_paged_attention_scatter``) must leave the same
pool bytes and return the same rows as ``write_layer`` followed by ``attend_layer`` (bit
for bit: the same copy and the same attention math), including new rows that straddle a
split boundary, and match the oracle within the bf16/f16 tolerance (2e-2). Shapes the
decode kernel does not take run the two kernels in turn.
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


def twins(lengths, query_len, dtype, seed, split, page_size=128):
    """Two managers with identical pools and histories, and one step's inputs."""
    pages = sum(math.ceil((n + query_len) / page_size) for n in lengths) + 2
    out = []
    for _ in range(2):
        gen = torch.Generator(device="cuda").manual_seed(seed)
        m = PagedKVCacheManager(2, 8, 128, pages * page_size, page_size, len(lengths), dtype, "cuda")
        m.split_tokens = split
        W.shuffle_free_pages(m, seed)
        hs = [m.allocate() for _ in lengths]
        for h, n in zip(hs, lengths):
            W.fill_history(m, h, n, gen, layers=[1])
        out.append((m, hs))
    gen = torch.Generator(device="cuda").manual_seed(seed + 7)
    q, k, v = W.step_inputs(out[0][0], out[0][1], query_len, 32, gen)
    return out, q, k, v


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
@pytest.mark.parametrize("query_len", [1, 2, 4])
@pytest.mark.parametrize("split", [0, 64, 192])
def test_fused_step_equals_write_then_attend(dtype, query_len, split):
    # 63 / 127 / 191 put multi-token steps across a 64-token split boundary
    lengths = [0, 1, 63, 127, 191, 1000, 2431]
    ((ma, ha), (mb, hb)), q, k, v = twins(lengths, query_len, dtype, seed=query_len + split, split=split)
    fused = ma.begin_batch(ha, query_len).write_attend_layer(1, k, v, q)
    batch = mb.begin_batch(hb, query_len)
    batch.write_layer(1, k, v)
    ref = batch.attend_layer(q, 1)
    torch.cuda.synchronize()
    ma.check_device_errors()
    mb.check_device_errors()
    assert torch.equal(ma.k_cache, mb.k_cache) and torch.equal(ma.v_cache, mb.v_cache)
    assert torch.equal(fused, ref)
    kp, vp = ma.k_cache.float().cpu().numpy(), ma.v_cache.float().cpu().numpy()
    table = np.full((len(ha), max(len(h.pages) for h in ha)), -1, dtype=np.int64)
    for i, h in enumerate(ha):
        table[i, :len(h.pages)] = h.pages
    lens = np.asarray([h.length for h in ha], dtype=np.int64)
    exp = oracle.paged_attention(q.float().cpu().numpy(), kp, vp, 1, table, lens, ma.page_size)
    assert np.abs(fused.float().cpu().numpy() - exp).max() <= 2e-2


def test_fused_step_commits_like_write_layer():
    """Several fused steps in a row: each step's rows land where the next one reads them."""
    ((ma, ha), (mb, hb)), _, _, _ = twins([5, 300, 900], 1, torch.bfloat16, seed=3, split=64)
    gen = torch.Generator(device="cuda").manual_seed(11)
    for _ in range(5):
        q, k, v = W.step_inputs(ma, ha, 1, 32, gen)
        a = ma.begin_batch(ha, 1).write_attend_layer(1, k, v, q)
        batch = mb.begin_batch(hb, 1)
        batch.write_layer(1, k, v)
        b = batch.attend_layer(q, 1)
        ma.commit_batch(ha, 1)
        mb.commit_batch(hb, 1)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
    assert torch.equal(ma.k_cache, mb.k_cache) and torch.equal(ma.v_cache, mb.v_cache)


def test_unfused_shapes_run_both_kernels():
    """fp32 (no decode kernel) and a prefill-size chunk take the two-kernel path."""
    for dtype, query_len in ((torch.float32, 1), (torch.bfloat16, 40)):
        ((ma, ha), (mb, hb)), q, k, v = twins([100, 700], query_len, dtype, seed=5, split=0)
        fused = ma.begin_batch(ha, query_len).write_attend_layer(1, k, v, q)
        batch = mb.begin_batch(hb, query_len)
        batch.write_layer(1, k, v)
        ref = batch.attend_layer(q, 1)
        torch.cuda.synchronize()
        assert torch.equal(ma.k_cache, mb.k_cache) and torch.equal(ma.v_cache, mb.v_cache)
        assert torch.equal(fused, ref)


def test_fused_step_refuses_bad_page():
    """A new row's page id outside the pool: flagged, and that split writes nothing."""
    ((ma, ha), _), q, k, v = twins([300], 1, torch.bfloat16, seed=9, split=0)
    batch = ma.begin_batch(ha, 1)
    table = batch.page_table.clone()
    table[0, 2] = ma.num_pages + 3  # position 300 sits on page 2
    before = ma.k_cache.clone()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    workspace = ma.workspace_for(1, 1, 32, batch.max_kv_len)
    ops.paged_attention_scatter(q, k, v, ma.k_cache, ma.v_cache, 1, table, batch.cache_lens_i32,
                                ma.page_size, batch.max_kv_len, workspace=workspace, error_word=err)
    torch.cuda.synchronize()
    assert "page id outside the pool" in ops.read_device_errors(err)
    assert torch.equal(ma.k_cache, before)
