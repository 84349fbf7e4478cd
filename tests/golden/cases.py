"""Golden parity cases shared by ``make_golden.py`` and the tests.

Every input value is ``k / 64`` with ``k`` the sum of two integers drawn from
``[-64, 64)`` by ``numpy.random.RandomState`` (a frozen stream), optionally
times a power of two. These values are exact in bf16, fp16 and fp32, so the
reference's fp32 CPU run, the oracle and the bf16 CUDA kernels all see
bit-identical inputs, and the generator needs no transcendental function whose
last bit could differ between hosts.

A case describes one ``begin_batch(handles, T)`` → ``write_layer`` →
``attend_layer`` step of ``hayate/engine/paged_cache.py:202-293,44-71``: each
request first imports ``history`` tokens of K/V into its pages
(``allocate_for_request``, ``paged_cache.py:142-166``), then ``T`` new tokens
are written and attended. The manager's free-page stack is shuffled with
``random.Random(seed)`` so page tables are non-contiguous.
"""

from __future__ import annotations

import random
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Case:
    name: str
    num_layers: int
    layer: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    page_size: int
    max_cache_tokens: int
    history: tuple[int, ...]
    query_len: int
    seed: int
    q_scale: float = 1.0

    @property
    def batch(self) -> int:
        return len(self.history)


CASES = (
    # The reference's own CUDA parity test shapes (tests/test_paged_cache.py:58-93):
    # H_q=4, H_kv=2, D=16, page 128, histories 130 and 200, T=2, seed 23.
    Case("ref_test_shape", 1, 0, 4, 2, 16, 128, 1024, (130, 200), 2, 23),
    # Qwen3-4B heads, decode T=1; histories end on, just before and past a page edge.
    Case("qwen_decode", 1, 0, 32, 8, 128, 128, 2048, (127, 128, 300, 1), 1, 5),
    # Qwen3-4B heads, a ragged prefill chunk on top of an empty and a 200-token prefix,
    # with sharper scores (q scaled by 8) to exercise the running max.
    Case("qwen_prefill", 1, 0, 32, 8, 128, 128, 2048, (0, 200), 9, 7, 8.0),
    # Two layers (writes land in layer 1 only), page 256, head_dim 64, group of 4.
    Case("multi_layer_page256", 2, 1, 8, 2, 64, 256, 4096, (0, 255, 513), 3, 11),
    # No grouping (H_q == H_kv), head_dim 32, a 130-token chunk crossing two page edges.
    Case("mha_long_chunk", 1, 0, 2, 2, 32, 128, 1024, (5,), 130, 13),
)


# Cases run through the reference's own GPU path (its torch.compile'd FlexAttention, bf16)
# by ``make_reference_gpu.py`` on a B200; the tests compare this repository's kernels with
# the stored rows on boxes where the reference is not installed.
GPU_CASES = (
    # decode, ragged histories across page edges (one split and several per request)
    Case("refgpu_decode", 1, 0, 32, 8, 128, 128, 8192, (1000, 4095, 129, 2048), 1, 31),
    # four new tokens per request: the decode kernel's 16-row tile (4 heads x 4 tokens)
    Case("refgpu_decode_t4", 1, 0, 32, 8, 128, 128, 2048, (127, 128, 300, 1), 4, 37),
    # a prefill chunk over an empty, a short and a long prefix
    Case("refgpu_prefill", 1, 0, 32, 8, 128, 128, 4096, (0, 300, 1500), 40, 41),
    # a long and a short prefix, a chunk crossing a page edge, sharper scores (two requests:
    # the reference's compiled FlexAttention fails to lower for a one-request batch on B200,
    # Inductor NoValidChoicesError)
    Case("refgpu_prefill_long", 1, 0, 32, 8, 128, 128, 4096, (2500, 700), 64, 43, 4.0),
)


def case_by_name(name: str) -> Case:
    for case in CASES + GPU_CASES:
        if case.name == name:
            return case
    raise KeyError(name)


def exact_values(rs: np.random.RandomState, shape, scale: float = 1.0) -> np.ndarray:
    """Triangular values ``(a + b) / 64`` with ``a, b`` uniform in ``[-64, 64)``; exact in bf16."""
    a = rs.randint(-64, 64, size=shape).astype(np.int64)
    b = rs.randint(-64, 64, size=shape).astype(np.int64)
    return ((a + b).astype(np.float32) / np.float32(64.0)) * np.float32(scale)


def make_inputs(case: Case) -> dict:
    """Regenerate the inputs of a case: per-request history K/V and the step's q, k, v."""
    rs = np.random.RandomState(case.seed)
    hist_k, hist_v = [], []
    for length in case.history:
        hist_k.append(exact_values(rs, (case.num_layers, case.num_kv_heads, length, case.head_dim)))
        hist_v.append(exact_values(rs, (case.num_layers, case.num_kv_heads, length, case.head_dim)))
    B, T = case.batch, case.query_len
    q = exact_values(rs, (B, case.num_q_heads, T, case.head_dim), case.q_scale)
    k_new = exact_values(rs, (B, case.num_kv_heads, T, case.head_dim))
    v_new = exact_values(rs, (B, case.num_kv_heads, T, case.head_dim))
    return {"hist_k": hist_k, "hist_v": hist_v, "q": q, "k_new": k_new, "v_new": v_new}


def shuffled_free_pages(num_pages: int, seed: int) -> list[int]:
    """The free-page stack (popped from the end) after a seeded shuffle."""
    pages = list(range(num_pages - 1, -1, -1))
    random.Random(seed).shuffle(pages)
    return pages
