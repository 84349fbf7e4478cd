"""Packed (mixed prefill + decode) batches on the GPU.

One packed step (``begin_batch(handles, [T_0, T_1, ...])``) must write the same pool
bytes and produce the same attention rows as running each request on its own with the
uniform path (bit for bit: the same kernels serve each request), and match the oracle
within the usual tolerances (2e-2 bf16/f16, 1e-4 f32).
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

TOL = {torch.bfloat16: 2e-2, torch.float16: 2e-2, torch.float32: 1e-4}
MIXED = ([0, 5, 1000, 130, 4095, 17, 256], [1, 37, 1, 300, 1, 128, 2])


def twin_managers(lengths, query_lens, dtype, seed, page_size=128):
    """Two managers with identical pools, page assignments and histories."""
    pages = sum(math.ceil((n + t) / page_size) for n, t in zip(lengths, query_lens)) + 2
    out = []
    for _ in range(2):
        gen = torch.Generator(device="cuda").manual_seed(seed)
        m = PagedKVCacheManager(1, 8, 128, pages * page_size, page_size, len(lengths), dtype, "cuda")
        m.split_tokens = 256
        m.prefill_plan = False  # the default grid: bit-exact with the per-request launches
        W.shuffle_free_pages(m, seed)
        hs = [m.allocate() for _ in lengths]
        for h, n in zip(hs, lengths):
            W.fill_history(m, h, n, gen)
        out.append((m, hs))
    return out


def packed_inputs(query_lens, dtype, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed + 1)
    n = sum(query_lens)
    q = torch.randn(1, n, 32, 128, generator=gen, device="cuda").to(dtype).transpose(1, 2)
    k = torch.randn(1, n, 8, 128, generator=gen, device="cuda").to(dtype).transpose(1, 2)
    v = torch.randn(1, n, 8, 128, generator=gen, device="cuda").to(dtype).transpose(1, 2)
    return q, k, v


def per_request(m, hs, query_lens, q, k, v):
    """The uniform path, one request at a time; rows concatenated on the token axis."""
    rows = []
    start = 0
    for h, t in zip(hs, query_lens):
        batch = m.begin_batch([h], t)
        sl = slice(start, start + t)
        batch.write_layer(0, k[:, :, sl], v[:, :, sl])
        m.kernel = "decode" if t == 1 and m.k_cache.dtype != torch.float32 else (
            "prefill" if m.k_cache.dtype != torch.float32 else "generic")
        rows.append(batch.attend_layer(q[:, :, sl], 0))
        start += t
    m.kernel = "auto"
    return torch.cat(rows, dim=2)


def oracle_rows(m, hs, query_lens, q):
    kp = m.k_cache.float().cpu().numpy()
    vp = m.v_cache.float().cpu().numpy()
    rows, start = [], 0
    for h, t in zip(hs, query_lens):
        table = np.asarray([h.pages], dtype=np.int64)
        lens = np.asarray([h.length], dtype=np.int64)
        qb = q[:, :, start:start + t].float().cpu().numpy()
        rows.append(oracle.paged_attention(qb, kp, vp, 0, table, lens, m.page_size))
        start += t
    return np.concatenate(rows, axis=2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32], ids=str)
@pytest.mark.parametrize("lengths, query_lens", [
    MIXED,
    ([3000, 10, 700], [1, 1, 1]),          # decode only
    ([0, 129, 2000], [513, 64, 129]),      # prefill only
    ([64], [5]),
], ids=["mixed", "decode_only", "prefill_only", "single"])
def test_packed_step_equals_per_request_steps(lengths, query_lens, dtype):
    (ma, ha), (mb, hb) = twin_managers(lengths, query_lens, dtype, seed=sum(query_lens))
    q, k, v = packed_inputs(query_lens, dtype, seed=len(lengths))
    batch = ma.begin_batch(ha, query_lens)
    assert batch.layout is not None and batch.layout.total_tokens == sum(query_lens)
    batch.write_layer(0, k, v)
    out = batch.attend_layer(q, 0)
    ref = per_request(mb, hb, query_lens, q, k, v)
    torch.cuda.synchronize()
    ma.check_device_errors()
    mb.check_device_errors()
    assert torch.equal(ma.k_cache, mb.k_cache) and torch.equal(ma.v_cache, mb.v_cache)
    assert out.shape == q.shape and out.transpose(1, 2).is_contiguous()
    assert torch.equal(out, ref)
    err = np.abs(out.float().cpu().numpy() - oracle_rows(ma, ha, query_lens, q)).max()
    assert err <= TOL[dtype], err


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
def test_packed_prepare_layer_equals_per_request(dtype):
    lengths, query_lens = MIXED
    (ma, ha), (mb, hb) = twin_managers(lengths, query_lens, dtype, seed=7)
    gen = torch.Generator(device="cuda").manual_seed(3)
    n = sum(query_lens)
    q = torch.randn(1, n, 32, 128, generator=gen, device="cuda").to(dtype)
    k = torch.randn(1, n, 8, 128, generator=gen, device="cuda").to(dtype)
    v = torch.randn(1, n, 8, 128, generator=gen, device="cuda").to(dtype)
    wq = (1 + 0.1 * torch.randn(128, generator=gen, device="cuda")).to(dtype)
    wk = (1 + 0.1 * torch.randn(128, generator=gen, device="cuda")).to(dtype)
    cos, sin = W.rope_angles(torch.arange(8192, device="cuda"), 128)
    cos, sin = cos.contiguous(), sin.contiguous()
    q_packed = ma.begin_batch(ha, query_lens).prepare_layer(0, q, k, v, wq, wk, cos, sin)
    rows, start = [], 0
    for h, t in zip(hb, query_lens):
        sl = slice(start, start + t)
        rows.append(mb.begin_batch([h], t).prepare_layer(0, q[:, sl], k[:, sl], v[:, sl], wq, wk, cos, sin))
        start += t
    torch.cuda.synchronize()
    ma.check_device_errors()
    assert torch.equal(q_packed, torch.cat(rows, dim=2))
    assert torch.equal(ma.k_cache, mb.k_cache) and torch.equal(ma.v_cache, mb.v_cache)


def test_packed_commit_advances_each_request_by_its_own_length():
    lengths, query_lens = MIXED
    (ma, ha), _ = twin_managers(lengths, query_lens, torch.bfloat16, seed=1)
    ma.begin_batch(ha, query_lens)
    ma.commit_batch(ha, query_lens)
    assert [h.length for h in ha] == [n + t for n, t in zip(lengths, query_lens)]


def test_packed_metadata_out_of_range_is_flagged():
    """A q_len beyond the launch's longest chunk is refused on the device, not read."""
    lengths, query_lens = MIXED
    (ma, ha), _ = twin_managers(lengths, query_lens, torch.bfloat16, seed=2)
    q, k, v = packed_inputs(query_lens, torch.bfloat16, seed=2)
    batch = ma.begin_batch(ha, query_lens)
    batch.write_layer(0, k, v)
    lay = batch.layout
    bad_len = lay.q_len.clone()
    bad_len[int(lay.prefill_ids[0].item())] = max(query_lens) + 1
    ops.paged_attention_packed(q, ma.k_cache, ma.v_cache, 0, batch.page_table, batch.cache_lens_i32,
                               lay.q_start, bad_len, lay.decode_ids, lay.prefill_ids, ma.page_size,
                               batch.query_len, batch.max_kv_len,
                               workspace=ma.workspace_for(lay.decode_ids.numel(), 1, 32, batch.max_kv_len),
                               error_word=ma.error_word, split_tokens=256)
    torch.cuda.synchronize()
    assert "packed batch metadata (q_start / q_len / request id) out of range" in ops.read_device_errors(ma.error_word)
    ma.error_word.zero_()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=str)
def test_packed_step_with_prefill_schedule(dtype):
    """The packed batch's prefill launch on a plan (its prefill requests, in prefill_ids
    order) gives the default grid's rows within 2e-2 and the oracle's."""
    lengths, query_lens = [0, 5, 9000, 130, 4095, 17, 2560], [1, 37, 300, 300, 1, 128, 600]
    (ma, ha), (mb, hb) = twin_managers(lengths, query_lens, dtype, seed=11)
    ma.prefill_plan = True
    q, k, v = packed_inputs(query_lens, dtype, seed=4)
    batch = ma.begin_batch(ha, query_lens)
    planned = batch.prefill_schedule(q)
    assert planned is not None  # this mix of chunks is scheduled
    batch.write_layer(0, k, v)
    out = batch.attend_layer(q, 0)
    ref_batch = mb.begin_batch(hb, query_lens)
    ref_batch.write_layer(0, k, v)
    ref = ref_batch.attend_layer(q, 0)
    torch.cuda.synchronize()
    ma.check_device_errors()
    assert (out.float() - ref.float()).abs().max().item() <= 2e-2
    err = np.abs(out.float().cpu().numpy() - oracle_rows(ma, ha, query_lens, q)).max()
    assert err <= TOL[dtype], err
