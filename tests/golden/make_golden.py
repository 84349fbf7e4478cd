"""Generate golden vectors by running the unmodified hayate reference on CPU.

Usage::

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <hayate-exp checkout>

For every case in ``cases.py`` this drives the reference's own
``PagedKVCacheManager`` (``hayate/engine/paged_cache.py:74-304``) in fp32 on the
CPU: ``allocate_for_request`` imports each request's history, ``begin_batch``
reserves the append pages and builds the page table, ``write_layer`` scatters
the new K/V and ``attend_layer`` runs FlexAttention. ``torch.compile`` of
FlexAttention does not lower on the CPU with torch 2.11, so the module-level
``_compiled_flex_attention`` (``paged_cache.py:20``) is replaced by the eager
``flex_attention``; the attention math and masks are the reference's own.

Saved per case (``<name>.npz``): the page table and lengths the reference
built, the attention output, the set of pool slots the write changed, and a
SHA-256 of each pool's bytes after the write (pools start zeroed).
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from cases import CASES, make_inputs, shuffled_free_pages  # noqa: E402


def pool_digest(pool) -> str:
    return hashlib.sha256(np.ascontiguousarray(pool, dtype=np.float32).tobytes()).hexdigest()


def run_case(case, torch, paged_cache, Cache):
    inputs = make_inputs(case)
    manager = paged_cache.PagedKVCacheManager(
        num_layers=case.num_layers,
        num_kv_heads=case.num_kv_heads,
        head_dim=case.head_dim,
        max_cache_tokens=case.max_cache_tokens,
        page_size=case.page_size,
        max_requests=case.batch,
        dtype=torch.float32,
        device="cpu",
    )
    manager.k_cache.zero_()
    manager.v_cache.zero_()
    manager._free_pages = shuffled_free_pages(manager.num_pages, case.seed)
    handles = []
    for hk, hv in zip(inputs["hist_k"], inputs["hist_v"]):
        cache = Cache.from_tensors(torch.from_numpy(hk), torch.from_numpy(hv)) if hk.shape[2] else None
        handles.append(manager.allocate_for_request(cache))
    batch = manager.begin_batch(handles, case.query_len)
    before_k = manager.k_cache.clone()
    with torch.inference_mode():
        batch.write_layer(case.layer, torch.from_numpy(inputs["k_new"]), torch.from_numpy(inputs["v_new"]))
        out = batch.attend_layer(torch.from_numpy(inputs["q"]), case.layer)
    changed = (manager.k_cache[case.layer, 0] != before_k[case.layer, 0]).any(dim=-1).any(dim=0)
    return {
        "page_table": batch.page_table.numpy().astype(np.int64),
        "cache_lens": batch.cache_lens.numpy().astype(np.int64),
        "handle_pages": np.array([len(h.pages) for h in handles], dtype=np.int64),
        "out": out.float().numpy(),
        "changed_slots": np.nonzero(changed.numpy())[0].astype(np.int64),
        "k_pool_sha256": np.array(pool_digest(manager.k_cache.numpy())),
        "v_pool_sha256": np.array(pool_digest(manager.v_cache.numpy())),
    }


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="hayate-exp source checkout")
    parser.add_argument("--out", default=HERE)
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    from torch.nn.attention.flex_attention import flex_attention
    import hayate.engine.paged_cache as paged_cache
    from hayate.model.cache import Cache

    paged_cache._compiled_flex_attention = flex_attention
    torch.manual_seed(0)
    for case in CASES:
        result = run_case(case, torch, paged_cache, Cache)
        path = os.path.join(args.out, f"{case.name}.npz")
        np.savez_compressed(path, **result)
        print(f"{case.name}: out {result['out'].shape}, {len(result['changed_slots'])} slots written -> {path}")


if __name__ == "__main__":
    main()
