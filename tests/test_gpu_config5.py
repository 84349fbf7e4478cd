"""Config 5's shapes, reduced to two prefix groups on one GPU, against the oracle.

Config 5 is 512 requests with 32,768-token contexts in groups of 16 that alias one
4,096-token prefix (32 whole pages, shared through ``share``), decoding one token per
step. This test keeps every dimension of one request and of one group (32K contexts,
16-way aliasing of a 4K prefix, shuffled pages) and two groups instead of 32, plus two
forks that share all but the last few tokens of a group member: their first append lands
in a page the member still holds, so ``begin_batch`` copies that page first
(copy-on-write). Three decode steps run through ``write_attend_layer`` (one launch of the
decode kernel, which writes the step's rows itself) with ``commit_batch`` between them;
after the last one, sampled requests of both groups, both forks and the member whose
page was forked are compared with the oracle (max-abs 2e-2, bf16), every appended row is
checked bit for bit, and the page reference counts are checked.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from hayate_b200 import PagedKVCacheManager
from hayate_b200 import workloads as W

pytestmark = pytest.mark.gpu

GROUPS, PER_GROUP, PREFIX, CONTEXT, STEPS = 2, 16, 4096, 32768, 3
FORKS = ((0, 0, CONTEXT - 50), (1, 3, CONTEXT - 1))  # (group, member, shared tokens)


def oracle_rows(manager, batch, q, requests):
    """Oracle output rows for each request, on a compact copy of only its pages."""
    table = batch.page_table.cpu().numpy().astype(np.int64)
    lens = batch.cache_lens.cpu().numpy()
    P, H, D = manager.page_size, manager.num_kv_heads, manager.head_dim
    rows = {}
    for b in requests:
        n = -(-(int(lens[b]) + 1) // P)
        pages = torch.from_numpy(table[b, :n]).cuda()
        pools = [pool[0, 0].view(H, manager.num_pages, P, D).index_select(1, pages)
                 .reshape(1, 1, H, n * P, D).float().cpu().numpy()
                 for pool in (manager.k_cache, manager.v_cache)]
        rows[b] = oracle.paged_attention(q[b:b + 1].float().cpu().numpy(), pools[0], pools[1], 0,
                                         np.arange(n, dtype=np.int64)[None], lens[b:b + 1], P)[0]
    return rows


def test_reduced_config5_shared_prefixes_and_forks_match_oracle():
    gen = torch.Generator(device="cuda").manual_seed(5)
    own_pages = (CONTEXT - PREFIX) // 128
    pages = GROUPS * (PREFIX // 128 + PER_GROUP * (own_pages + 1)) + 2 * len(FORKS) + 16
    n_req = GROUPS * PER_GROUP + len(FORKS)
    m = PagedKVCacheManager(1, 8, 128, pages * 128, 128, n_req + GROUPS, torch.bfloat16, "cuda")
    W.shuffle_free_pages(m, 5)
    groups = []
    for _ in range(GROUPS):
        root = m.allocate()
        W.fill_history(m, root, PREFIX, gen)
        members = []
        for _ in range(PER_GROUP):
            h = m.share(root, PREFIX)                       # the prefix's 32 pages, aliased
            W.fill_history(m, h, CONTEXT, gen, start=PREFIX)
            members.append(h)
        m.release(root)                                     # the 16 members keep the pages
        groups.append(members)
    handles = [h for members in groups for h in members]
    forks = [m.share(groups[g][i], n) for g, i, n in FORKS]
    handles += forks
    prefix_pages = [members[0].pages[: PREFIX // 128] for members in groups]
    for g, ids in enumerate(prefix_pages):
        assert all(m.page_refcount(p) == PER_GROUP + sum(1 for f in FORKS if f[0] == g) for p in ids)

    forked_page = [groups[g][i].pages[n // 128] for g, i, n in FORKS]
    start_lens = [h.length for h in handles]
    written = []
    for step in range(STEPS):
        q, k, v = W.step_inputs(m, handles, 1, 32, gen)
        batch = m.begin_batch(handles, 1)
        if step == 0:  # the forks' first append copied the page they shared with their member
            for f, (g, i, n), old in zip(forks, FORKS, forked_page):
                assert f.pages[n // 128] != old and groups[g][i].pages[n // 128] == old
                assert m.page_refcount(old) == 1
        out = batch.write_attend_layer(0, k, v, q)
        torch.cuda.synchronize()
        m.check_device_errors()
        written.append((batch.page_table.long().clone(), batch.cache_lens.clone(), k, v))
        if step < STEPS - 1:
            m.commit_batch(handles, 1)

    # sampled requests of both groups, both forks and the members they forked, vs the oracle
    sample = sorted({0, 5, 15, PER_GROUP + 3, PER_GROUP + 9, 2 * PER_GROUP - 1,
                     FORKS[1][1] + PER_GROUP, n_req - 2, n_req - 1})
    assert len(sample) >= 8
    ref = oracle_rows(m, batch, q, sample)
    got = out.float().cpu().numpy()
    err = max(float(np.abs(got[b] - ref[b]).max()) for b in sample)
    assert err <= 2e-2, err

    # every step's new rows sit at their slots, bit for bit (nothing overwrote them later)
    m.commit_batch(handles, 1)
    rows = torch.arange(n_req, device="cuda")
    for table, lens, k, v in written:
        slots = table[rows, lens // 128] * 128 + lens % 128
        assert torch.equal(m.k_cache[0, 0][:, slots], k[:, :, 0].transpose(0, 1))
        assert torch.equal(m.v_cache[0, 0][:, slots], v[:, :, 0].transpose(0, 1))
    assert [h.length for h in handles] == [n + STEPS for n in start_lens]
    # the forks' private copy carries the member's rows before the fork point
    for f, (g, i, n) in zip(forks, FORKS):
        first = (n // 128) * 128
        pos = torch.arange(first, n, device="cuda")
        mine = torch.tensor(f.pages, device="cuda")[pos // 128] * 128 + pos % 128
        theirs = torch.tensor(groups[g][i].pages, device="cuda")[pos // 128] * 128 + pos % 128
        assert torch.equal(m.k_cache[0, 0][:, mine], m.k_cache[0, 0][:, theirs])
