"""Our kernels against the reference's own GPU attention (torch.compile'd FlexAttention).

Two forms. Live, where the reference is installed in ``baseline/_ref`` (an offline pip
install of hayate-exp): inputs go through the reference's own ``allocate_for_request``/
``begin_batch``/``write_layer``/``attend_layer`` on this GPU (its pools zeroed first: it
allocates them with ``torch.empty``). Recorded, everywhere: the same reference path was
run on a B200 by ``tests/golden/make_reference_gpu.py`` on exact-valued inputs, and its
rows, page tables and pool digests are fixtures in ``tests/golden/refgpu_*.npz``.
"""

from __future__ import annotations

import math
import os
import sys

import pytest
import torch

from golden_util import GPU_CASES, load_golden, make_inputs, shuffled_free_pages
from hayate_b200 import KVSnapshot, PagedKVCacheManager
from hayate_b200 import workloads as W

pytestmark = pytest.mark.gpu

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF_DIR, "hayate")):
        pytest.skip("reference not installed in baseline/_ref")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import hayate.engine.paged_cache as paged_cache
    from hayate.model.cache import Cache

    return paged_cache, Cache


@pytest.mark.parametrize("lengths, query_len", [([1000, 4095, 129, 2048], 1), ([0, 300, 1500], 200)])
def test_matches_reference_gpu_attention(ref, lengths, query_len):
    paged_cache, Cache = ref
    gen = torch.Generator(device="cuda").manual_seed(query_len)
    pages = sum(math.ceil((n + query_len) / 128) for n in lengths) + 4
    ours = PagedKVCacheManager(1, 8, 128, pages * 128, 128, len(lengths), torch.bfloat16, "cuda")
    W.shuffle_free_pages(ours, 2)
    hs = [ours.allocate() for _ in lengths]
    for h, n in zip(hs, lengths):
        W.fill_history(ours, h, n, gen)
    q, k, v = W.step_inputs(ours, hs, query_len, 32, gen)
    rm = paged_cache.PagedKVCacheManager(1, 8, 128, pages * 128, 128, len(lengths), torch.bfloat16, "cuda")
    rm.k_cache.zero_()
    rm.v_cache.zero_()
    rhs = []
    for h in hs:
        snap = ours.snapshot(h)
        rhs.append(rm.allocate_for_request(Cache.from_tensors(snap.k, snap.v) if h.length else None))
    rb = rm.begin_batch(rhs, query_len)
    ob = ours.begin_batch(hs, query_len)
    with torch.inference_mode():
        rb.write_layer(0, k.contiguous(), v.contiguous())
        expected = rb.attend_layer(q.contiguous(), 0)
    ob.write_layer(0, k, v)
    got = ob.attend_layer(q, 0)
    torch.cuda.synchronize()
    ours.check_device_errors()
    assert (got.float() - expected.float()).abs().max().item() <= 2e-2


def _bf16_digest(t: torch.Tensor) -> str:
    import hashlib

    return hashlib.sha256(t.contiguous().view(torch.int16).cpu().numpy().tobytes()).hexdigest()


@pytest.mark.parametrize("case", GPU_CASES, ids=lambda c: c.name)
def test_matches_recorded_reference_gpu_rows(case):
    """The reference's GPU rows recorded on a B200: same page tables, bit-equal pools after
    the write, attention within 2e-2."""
    golden = load_golden(case.name)
    inputs = make_inputs(case)
    dev = lambda a: torch.from_numpy(a).to("cuda", torch.bfloat16)  # noqa: E731
    m = PagedKVCacheManager(case.num_layers, case.num_kv_heads, case.head_dim, case.max_cache_tokens,
                            case.page_size, case.batch, torch.bfloat16, "cuda")
    m._free_pages = shuffled_free_pages(m.num_pages, case.seed)
    hs = [m.allocate_for_request(KVSnapshot(dev(hk), dev(hv)) if hk.shape[2] else None)
          for hk, hv in zip(inputs["hist_k"], inputs["hist_v"])]
    batch = m.begin_batch(hs, case.query_len)
    batch.write_layer(case.layer, dev(inputs["k_new"]), dev(inputs["v_new"]))
    out = batch.attend_layer(dev(inputs["q"]), case.layer)
    torch.cuda.synchronize()
    m.check_device_errors()
    table = golden["page_table"]
    width = batch.page_table.shape[1]
    assert (batch.page_table.cpu().numpy() == table[:, :width]).all() and (table[:, width:] == -1).all()
    assert (batch.cache_lens.cpu().numpy() == golden["cache_lens"]).all()
    assert _bf16_digest(m.k_cache) == str(golden["k_pool_sha256"])
    assert _bf16_digest(m.v_cache) == str(golden["v_pool_sha256"])
    expected = torch.from_numpy(golden["out_bf16"]).view(torch.bfloat16).float()
    err = (out.float().cpu() - expected).abs().max().item()
    assert err <= 2e-2, err
