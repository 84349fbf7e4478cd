"""Helpers to load the golden cases and rebuild their pools (shared by the tests)."""

from __future__ import annotations

import hashlib
import math
import os
import sys

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
if GOLDEN_DIR not in sys.path:
    sys.path.insert(0, GOLDEN_DIR)

from cases import CASES, GPU_CASES, case_by_name, make_inputs, shuffled_free_pages  # noqa: E402,F401


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN_DIR, f"{name}.npz")) as data:
        return {key: data[key] for key in data.files}


def pool_shape(case) -> tuple[int, ...]:
    num_pages = math.ceil(case.max_cache_tokens / case.page_size)
    return (case.num_layers, 1, case.num_kv_heads, num_pages * case.page_size, case.head_dim)


def history_pools(case, inputs: dict, page_table: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Zeroed fp32 pools holding each request's imported history at its paged slots.

    The import mirrors ``allocate_for_request``/``import_cache`` of the reference
    (``hayate/engine/paged_cache.py:142-166``): every layer of the history is copied.
    """
    k_pool = np.zeros(pool_shape(case), dtype=np.float32)
    v_pool = np.zeros_like(k_pool)
    for b, (hk, hv) in enumerate(zip(inputs["hist_k"], inputs["hist_v"])):
        length = hk.shape[2]
        if not length:
            continue
        logical = np.arange(length)
        slots = page_table[b][logical // case.page_size] * case.page_size + logical % case.page_size
        for layer in range(case.num_layers):
            k_pool[layer, 0][:, slots, :] = hk[layer]
            v_pool[layer, 0][:, slots, :] = hv[layer]
    return k_pool, v_pool


def sha256_f32(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array, dtype=np.float32).tobytes()).hexdigest()
