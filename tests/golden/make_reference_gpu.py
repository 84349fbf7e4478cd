"""Record the reference's own GPU attention rows as fixtures (run on a B200).

Usage (from the repository root, with hayate-exp installed into ``baseline/_ref``)::

    python tests/golden/make_reference_gpu.py [--reference baseline/_ref] [--out tests/golden]

For every case in ``cases.GPU_CASES`` this drives the UNMODIFIED reference on the GPU in
bf16: its ``PagedKVCacheManager`` (``hayate/engine/paged_cache.py:74-304``) with the
free-page stack shuffled as the case says and the pools zeroed (the reference allocates
them with ``torch.empty``), ``allocate_for_request`` importing each history
(``:142-166``), ``begin_batch`` (``:202-293``), ``write_layer`` (``:44-60``) and
``attend_layer`` (``:62-71``), whose FlexAttention is the module's
``torch.compile(flex_attention, dynamic=True)`` (``:20``), i.e. the Triton kernel
Inductor generates on this GPU. Inputs are the case's exact values (``cases.make_inputs``),
so every path sees bit-identical bf16 inputs.

Saved per case (``<name>.npz``): the attention rows as bf16 bit patterns, the page table
and cache lengths the reference built, and the SHA-256 of each pool's bf16 bytes after the
write. ``tests/test_gpu_vs_reference_gpu.py`` compares this repository's kernels with them.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)

from cases import GPU_CASES, make_inputs, shuffled_free_pages  # noqa: E402


def bf16_digest(tensor) -> str:
    import torch

    return hashlib.sha256(tensor.contiguous().view(torch.int16).cpu().numpy().tobytes()).hexdigest()


def run_case(case, torch, paged_cache, Cache):
    inputs = make_inputs(case)
    dev = lambda a: torch.from_numpy(a).to("cuda", torch.bfloat16)  # noqa: E731
    manager = paged_cache.PagedKVCacheManager(
        num_layers=case.num_layers, num_kv_heads=case.num_kv_heads, head_dim=case.head_dim,
        max_cache_tokens=case.max_cache_tokens, page_size=case.page_size, max_requests=case.batch,
        dtype=torch.bfloat16, device="cuda")
    manager.k_cache.zero_()
    manager.v_cache.zero_()
    manager._free_pages = shuffled_free_pages(manager.num_pages, case.seed)
    handles = []
    for hk, hv in zip(inputs["hist_k"], inputs["hist_v"]):
        cache = Cache.from_tensors(dev(hk), dev(hv)) if hk.shape[2] else None
        handles.append(manager.allocate_for_request(cache))
    batch = manager.begin_batch(handles, case.query_len)
    with torch.inference_mode():
        batch.write_layer(case.layer, dev(inputs["k_new"]), dev(inputs["v_new"]))
        out = batch.attend_layer(dev(inputs["q"]), case.layer)
    torch.cuda.synchronize()
    return {
        "out_bf16": out.contiguous().view(torch.int16).cpu().numpy(),
        "page_table": batch.page_table.cpu().numpy().astype(np.int64),
        "cache_lens": batch.cache_lens.cpu().numpy().astype(np.int64),
        "k_pool_sha256": np.array(bf16_digest(manager.k_cache)),
        "v_pool_sha256": np.array(bf16_digest(manager.v_cache)),
        "torch_version": np.array(torch.__version__),
        "device": np.array(torch.cuda.get_device_name()),
    }


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.path.join(ROOT, "baseline", "_ref"),
                        help="directory holding the installed hayate package")
    parser.add_argument("--out", default=HERE)
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    import hayate.engine.paged_cache as paged_cache
    from hayate.model.cache import Cache

    if not torch.cuda.is_available():
        raise SystemExit("needs a CUDA GPU: the fixtures record the reference's GPU kernels")
    failed = []
    for case in GPU_CASES:
        try:
            result = run_case(case, torch, paged_cache, Cache)
        except Exception as exc:  # a shape the reference's compiled path cannot lower
            failed.append(case.name)
            print(f"{case.name}: the reference failed: {type(exc).__name__}: {str(exc).splitlines()[0][:300]}")
            continue
        path = os.path.join(args.out, f"{case.name}.npz")
        np.savez_compressed(path, **result)
        print(f"{case.name}: out {result['out_bf16'].shape} -> {path}")
    if failed:
        raise SystemExit(f"no fixture for {failed}")


if __name__ == "__main__":
    main()
