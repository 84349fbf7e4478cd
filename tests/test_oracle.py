"""Pin the CPU oracle against golden vectors produced by the reference itself."""

from __future__ import annotations

import numpy as np
import pytest

from golden_util import CASES, history_pools, load_golden, make_inputs, sha256_f32

import oracle


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_oracle_scatter_is_bit_exact_with_reference(case):
    golden = load_golden(case.name)
    inputs = make_inputs(case)
    k_pool, v_pool = history_pools(case, inputs, golden["page_table"])
    slots = oracle.kv_scatter(k_pool, v_pool, case.layer, inputs["k_new"], inputs["v_new"],
                              golden["page_table"], golden["cache_lens"], case.page_size)
    np.testing.assert_array_equal(np.sort(slots.reshape(-1)), golden["changed_slots"])
    assert sha256_f32(k_pool) == str(golden["k_pool_sha256"])
    assert sha256_f32(v_pool) == str(golden["v_pool_sha256"])


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_oracle_attention_matches_reference(case, dtype):
    golden = load_golden(case.name)
    inputs = make_inputs(case)
    k_pool, v_pool = history_pools(case, inputs, golden["page_table"])
    oracle.kv_scatter(k_pool, v_pool, case.layer, inputs["k_new"], inputs["v_new"],
                      golden["page_table"], golden["cache_lens"], case.page_size)
    out = oracle.paged_attention(inputs["q"], k_pool, v_pool, case.layer, golden["page_table"],
                                 golden["cache_lens"], case.page_size, dtype=dtype)
    # fp32 tolerance of the attention parity bar
    np.testing.assert_allclose(out, golden["out"], rtol=0, atol=1e-4)


def test_oracle_rejects_unreserved_page():
    table = np.array([[3, -1]], dtype=np.int64)
    with pytest.raises(ValueError):
        oracle.scatter_positions(table, np.array([127]), 2, 128)


def test_oracle_mutation_is_caught():
    """A planted off-by-one in the oracle's causal mask must break parity with the golden."""
    case = CASES[1]
    golden = load_golden(case.name)
    inputs = make_inputs(case)
    k_pool, v_pool = history_pools(case, inputs, golden["page_table"])
    oracle.kv_scatter(k_pool, v_pool, case.layer, inputs["k_new"], inputs["v_new"],
                      golden["page_table"], golden["cache_lens"], case.page_size)
    # drop the newest key from every request: attention over cache_len keys instead of cache_len + 1
    out = oracle.paged_attention(inputs["q"], k_pool, v_pool, case.layer, golden["page_table"],
                                 golden["cache_lens"] - 1 + (golden["cache_lens"] == 0), case.page_size)
    assert np.abs(out - golden["out"]).max() > 1e-2


def test_flops_and_bytes_formulas():
    # 4 * H_q * D per visible pair; decode bytes = kv_len * H_kv * D * 2 B * (K and V)
    assert oracle.attention_flops([0], 1, 32, 128) == 4 * 32 * 128
    assert oracle.attention_flops([10], 4, 1, 1) == 4 * (40 + 10)
    assert oracle.decode_bytes([512, 512], 8, 128) == 1024 * 8 * 128 * 2 * 2


def test_bench_flop_count_matches_the_oracle():
    """bench.py counts prefill FLOPs itself (its GPU legs do not touch oracle/)."""
    import bench

    for lens, t in (([2998, 4045, 1590, 2020, 1436, 3762, 183, 2532], 512), ([0], 1), ([5, 0, 77], 130)):
        assert bench.attention_flops(lens, t, 32, 128) == oracle.attention_flops(lens, t, 32, 128)
