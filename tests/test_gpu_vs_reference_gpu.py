"""Our kernels against the reference's own GPU attention (torch.compile'd FlexAttention).

Runs only where the reference is installed in ``baseline/_ref`` (an offline pip
install of hayate-exp); elsewhere the module is skipped. Inputs go through the
reference's own ``allocate_for_request``/``begin_batch``/``write_layer``/
``attend_layer``; its pools are zeroed first (it allocates them with torch.empty).
"""

from __future__ import annotations

import math
import os
import sys

import pytest
import torch

from hayate_b200 import PagedKVCacheManager
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
