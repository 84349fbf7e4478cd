"""The bounded pipeline wait runs out cleanly on the GPU.

Every mbarrier wait in the kernels gives up after 1 s, records the wait-timeout bit in
the error word and lets the CTA exit (``csrc/common.cuh``). Here a wait on a barrier
that nothing signals runs into that limit (no copy or tensor-core op is in flight);
the host must read the status, and the context must stay usable: a decode step right
after it matches the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from hayate_b200 import PagedKVCacheManager, ops
from hayate_b200 import workloads as W

import oracle

pytestmark = pytest.mark.gpu


def test_wait_runs_out_and_reports_timeout():
    error_word = torch.zeros(1, dtype=torch.int32, device="cuda")
    first, second = ops.wait_self_test(error_word)
    assert ops.read_device_errors(error_word) == ["a bounded pipeline wait gave up"], ops.read_device_errors(error_word)
    assert 1.0e9 <= first < 5.0e9, first      # the 1 s limit, not a hang
    assert second < 1.0e8, second              # later waits of the CTA return through its abort flag


def test_context_usable_after_timeout():
    error_word = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.wait_self_test(error_word)
    m = PagedKVCacheManager(1, 8, 128, 64 * 128, 128, 4, torch.bfloat16, "cuda")
    gen = torch.Generator(device="cuda").manual_seed(5)
    hs = [m.allocate() for _ in range(3)]
    for h, n in zip(hs, (700, 1, 2000)):
        W.fill_history(m, h, n, gen)
    q = torch.randn(3, 32, 1, 128, generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.randn(3, 8, 1, 128, generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn(3, 8, 1, 128, generator=gen, device="cuda").to(torch.bfloat16)
    batch = m.begin_batch(hs, 1)
    batch.write_layer(0, k, v)
    out = batch.attend_layer(q, 0)
    torch.cuda.synchronize()
    m.check_device_errors()
    kp, vp = m.k_cache.float().cpu().numpy(), m.v_cache.float().cpu().numpy()
    for b, h in enumerate(hs):
        ref = oracle.paged_attention(q[b:b + 1].float().cpu().numpy(), kp, vp, 0,
                                     np.asarray([h.pages], dtype=np.int64),
                                     np.asarray([h.length], dtype=np.int64), m.page_size)
        assert np.abs(out[b:b + 1].float().cpu().numpy() - ref).max() <= 2e-2
