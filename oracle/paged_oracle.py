"""NumPy restatement of hayate's paged KV write and paged attention.

TEST INFRASTRUCTURE, NOT PRODUCT CODE. This module is the checker the CUDA
kernels are compared against and the CPU baseline ``bench.py`` times. Nothing
in the ``hayate_b200`` package imports it.

What it restates (paths are inside the hayate-exp project):

* ``hayate/engine/paged_cache.py:44-60`` ``PagedKVBatch.write_layer``: the new
  token ``t`` of batch row ``b`` lives at logical position
  ``pos = cache_lens[b] + t``; its physical slot is
  ``page_table[b, pos // P] * P + pos % P`` and the write is
  ``pool[layer, 0, h, slot, :] = new[b, h, t, :]`` for K and for V.
* ``hayate/engine/paged_cache.py:62-71, 266-271, 358-374``
  ``PagedKVBatch.attend_layer``: FlexAttention with ``enable_gqa=True`` over the
  physical pool. A physical key is kept only if it maps back to a logical key
  ``j`` of the same request with ``j < kv_lens[b]`` and ``j <= cache_lens[b] + t``
  (``kv_lens = cache_lens + T``, ``paged_cache.py:217,255-256``); every other key
  gets a score of -inf. Physical keys therefore contribute exactly the logical
  keys ``0 .. cache_lens[b] + t`` of that request, which is what this oracle sums
  over after gathering them through the page table.
* FlexAttention defaults (torch ``nn/attention/flex_attention.py``, the torch
  2.10 pin of ``uv.lock:780-781``): softmax scale ``1/sqrt(D)``; with GQA the
  query head ``h`` reads KV head ``h // (H_q // H_kv)``.

Parity is pinned by ``tests/golden/*.npz``, produced by running the unmodified
reference ``PagedKVCacheManager`` / ``write_layer`` / ``attend_layer`` on CPU in
fp32 (``tests/golden/make_golden.py``) and checked in ``tests/test_oracle.py``.
"""

from __future__ import annotations

import math

import numpy as np


def scatter_positions(page_table: np.ndarray, cache_lens: np.ndarray, query_len: int,
                      page_size: int) -> np.ndarray:
    """Physical pool slot of every new token, shape ``[B, T]`` int64.

    Restates ``paged_cache.py:49-56``: logical position = ``cache_len + t``, page =
    ``pos // P`` looked up in the request's page table, slot = ``page * P + pos % P``.
    """
    page_table = np.asarray(page_table, dtype=np.int64)
    cache_lens = np.asarray(cache_lens, dtype=np.int64)
    logical = cache_lens[:, None] + np.arange(query_len, dtype=np.int64)[None, :]
    pages = np.take_along_axis(page_table, logical // page_size, axis=1)
    if (pages < 0).any():
        raise ValueError("a new token falls on an unreserved page (page id -1)")
    return pages * page_size + logical % page_size


def kv_scatter(k_pool: np.ndarray, v_pool: np.ndarray, layer: int, k_new: np.ndarray,
               v_new: np.ndarray, page_table: np.ndarray, cache_lens: np.ndarray,
               page_size: int) -> np.ndarray:
    """Write ``k_new``/``v_new`` ``[B, H_kv, T, D]`` into ``[L, 1, H_kv, cap, D]`` pools in place.

    Restates ``paged_cache.py:59-60``. Returns the ``[B, T]`` slots written.
    """
    B, H, T, D = k_new.shape
    slots = scatter_positions(page_table, cache_lens, T, page_size)
    flat = slots.reshape(-1)
    # pool[layer, 0, h, slot, :] = new[b, h, t, :]  (the reference permutes to [H, B, T, D])
    k_pool[layer, 0][:, flat, :] = np.transpose(k_new, (1, 0, 2, 3)).reshape(H, B * T, D)
    v_pool[layer, 0][:, flat, :] = np.transpose(v_new, (1, 0, 2, 3)).reshape(H, B * T, D)
    return slots


def _logical_slots(page_row: np.ndarray, length: int, page_size: int) -> np.ndarray:
    logical = np.arange(length, dtype=np.int64)
    pages = np.asarray(page_row, dtype=np.int64)[logical // page_size]
    if (pages < 0).any():
        raise ValueError("attended key falls on an unreserved page (page id -1)")
    return pages * page_size + logical % page_size


def paged_attention(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray, layer: int,
                    page_table: np.ndarray, cache_lens: np.ndarray, page_size: int,
                    scale: float | None = None, dtype=np.float32,
                    requests=None) -> np.ndarray:
    """Causal GQA attention over paged K/V, returning ``[B, H_q, T, D]``.

    ``q`` is ``[B, H_q, T, D]``; query ``t`` of row ``b`` attends logical keys
    ``0 .. cache_lens[b] + t`` (``paged_cache.py:266-271``). ``dtype`` is the
    accumulation type (fp32 like the reference's CPU run, or fp64 for a tighter
    check). ``requests`` optionally restricts the work to some batch rows (the
    bounded CPU-baseline sample); rows not computed are left as zeros.
    """
    B, Hq, T, D = q.shape
    Hkv = k_pool.shape[2]
    if Hq % Hkv:
        raise ValueError("query heads must be a multiple of KV heads")
    group = Hq // Hkv
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    out = np.zeros((B, Hq, T, D), dtype=dtype)
    rows = range(B) if requests is None else requests
    for b in rows:
        cache_len = int(cache_lens[b])
        kv_len = cache_len + T
        slots = _logical_slots(page_table[b], kv_len, page_size)
        k = k_pool[layer, 0][:, slots, :].astype(dtype, copy=False)   # [H_kv, kv_len, D]
        v = v_pool[layer, 0][:, slots, :].astype(dtype, copy=False)
        qb = q[b].astype(dtype, copy=False).reshape(Hkv, group * T, D)  # heads of a group share K/V
        s = np.matmul(qb, np.transpose(k, (0, 2, 1))) * dtype(scale)  # [H_kv, group*T, kv_len]
        s = s.reshape(Hkv, group, T, kv_len)
        # key j is visible to query t iff j <= cache_len + t (j < kv_len holds by construction)
        visible = np.arange(kv_len)[None, :] <= (cache_len + np.arange(T))[:, None]
        s = np.where(visible[None, None], s, -np.inf)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        o = np.matmul(p.reshape(Hkv, group * T, kv_len), v)  # [H_kv, group*T, D]
        out[b] = o.reshape(Hq, T, D)
    return out


def decode_bytes(kv_lens, num_kv_heads: int, head_dim: int, elem_bytes: int = 2) -> int:
    """Algorithmic HBM bytes of one paged-attention pass: every attended K and V row once."""
    return int(np.sum(np.asarray(kv_lens, dtype=np.int64))) * num_kv_heads * head_dim * elem_bytes * 2


def attention_flops(cache_lens, query_len: int, num_q_heads: int, head_dim: int) -> int:
    """Causal-valid attention FLOPs: 4 * H_q * D per visible (query, key) pair."""
    cache_lens = np.asarray(cache_lens, dtype=np.int64)
    pairs = np.sum(cache_lens * query_len + query_len * (query_len + 1) // 2)
    return int(pairs) * 4 * num_q_heads * head_dim
