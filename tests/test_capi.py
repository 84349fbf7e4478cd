"""The C ABI library loads, exports what include/hayate_b200.h declares, and
refuses bad arguments on the host (no GPU needed: every case returns before
any CUDA call)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from hayate_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "hayate_b200.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hyt_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) >= 9
    for name in names:
        assert hasattr(lib, name), name
    # the Python binding types every declared function
    assert set(names) == set(_lib.SIGNATURES)


def test_version_and_error_string():
    lib = _lib.lib()
    assert lib.hyt_version() == 100
    assert lib.hyt_last_error() == b""


def _scatter_args(**overrides):
    strides = _lib.int64_array([0] * 6)
    args = dict(k_new=1, v_new=1, strides=strides, k_pool=1, v_pool=1, num_layers=1, layer=0,
                capacity=1024, page_table=1, pts=8, cache_lens=1, batch=1, query_len=1, heads=8,
                head_dim=128, page_size=128, dtype=0, err=None, stream=None)
    args.update(overrides)
    return list(args.values())


@pytest.mark.parametrize("bad, message", [
    (dict(k_new=None), "null pointer"),
    (dict(batch=0), "batch"),
    (dict(query_len=0), "query_len"),
    (dict(page_size=96), "power of two"),
    (dict(capacity=1000), "multiple of page_size"),
    (dict(layer=1), "layer"),
    (dict(dtype=7), "dtype"),
])
def test_scatter_rejects_bad_arguments(bad, message):
    lib = _lib.lib()
    rc = lib.hyt_kv_scatter(*_scatter_args(**bad))
    assert rc == -1
    assert message in lib.hyt_last_error().decode()


def _attention_args(**overrides):
    s = _lib.int64_array([0, 0, 0])
    args = dict(q=1, qs=s, k_pool=1, v_pool=1, num_layers=1, layer=0, capacity=4096,
                page_table=1, pts=32, cache_lens=1, out=1, os=s, batch=2, query_len=1,
                hq=32, hkv=8, head_dim=128, page_size=128, dtype=0, scale=0.088,
                max_kv_len=4096, split_tokens=0, ws=None, ws_bytes=0, err=None, stream=None)
    args.update(overrides)
    return list(args.values())


@pytest.mark.parametrize("bad, code, message", [
    (dict(q=None), -1, "null pointer"),
    (dict(hq=30), -1, "multiple of num_kv_heads"),
    (dict(max_kv_len=0), -1, "max_kv_len"),
    (dict(split_tokens=-64), -1, "split_tokens"),
    (dict(max_kv_len=8192, ws=None), -4, "workspace"),
])
def test_attention_rejects_bad_arguments(bad, code, message):
    lib = _lib.lib()
    rc = lib.hyt_paged_attention(*_attention_args(**bad))
    assert rc == code
    assert message in lib.hyt_last_error().decode()


def test_decode_entry_refuses_unsupported_shape():
    lib = _lib.lib()
    rc = lib.hyt_decode_attention(*_attention_args(head_dim=64))
    assert rc == -2
    assert "head_dim 128" in lib.hyt_last_error().decode()


def test_generic_entry_refuses_unsupported_head_dim():
    lib = _lib.lib()
    args = _attention_args(head_dim=12)
    # the generic entry point has no split/workspace arguments
    args = args[:20] + args[24:]
    rc = lib.hyt_generic_attention(*args)
    assert rc == -2


def test_workspace_bytes_formula():
    lib = _lib.lib()
    # one split per (request, head) needs no workspace
    assert lib.hyt_attention_workspace_bytes(64, 1, 32, 8, 128, 512, 0, 0) == 0
    # forced 1024-token splits over 8192 keys: 8 splits x 4 rows
    units, splits, rows = 64 * 8, 8, 4
    expect = (((units * 4) + 255) // 256 * 256 + ((units * splits * rows * 2 * 4) + 255) // 256 * 256
              + units * splits * rows * 128 * 4)
    assert lib.hyt_attention_workspace_bytes(64, 1, 32, 8, 128, 8192, 1024, 0) == expect
    # f32 and head_dim 64 run on the CUDA-core kernel, which needs none
    assert lib.hyt_attention_workspace_bytes(64, 1, 32, 8, 128, 8192, 1024, 2) == 0
    assert lib.hyt_attention_workspace_bytes(64, 1, 32, 8, 64, 8192, 1024, 0) == 0


def test_workspace_init_accepts_empty():
    lib = _lib.lib()
    assert lib.hyt_workspace_init(None, 0, None) == 0
    assert lib.hyt_workspace_init(None, 16, None) == -1


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setenv("HAYATE_B200_LIB", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()
    monkeypatch.setattr(_lib, "_lib", None)


def test_ctypes_types_are_plain():
    # no torch types cross the boundary: every argument is a pointer or a scalar
    for restype, argtypes in _lib.SIGNATURES.values():
        for t in argtypes:
            assert t in (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t)


def _header_types():
    """ctypes type of every parameter of every declared function, from the header."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for name in declared_functions():
        params = re.search(r"\b" + name + r"\s*\((.*?)\);", text, re.S).group(1)
        types = []
        for a in (x.strip() for x in params.split(",")):
            if not a or a == "void":
                continue
            if "*" in a:
                types.append(ctypes.c_void_p)
            elif a.startswith("int64_t"):
                types.append(ctypes.c_int64)
            elif a.startswith("int32_t"):
                types.append(ctypes.c_int32)
            elif a.startswith("float"):
                types.append(ctypes.c_float)
            elif a.startswith("size_t"):
                types.append(ctypes.c_size_t)
            else:
                raise AssertionError(f"{name}: unexpected parameter {a!r}")
        out[name] = types
    return out


def test_binding_argument_types_match_the_header():
    for name, types in _header_types().items():
        assert list(_lib.SIGNATURES[name][1]) == types, name


def _packed_args(**overrides):
    s = _lib.int64_array([0, 0])
    args = dict(q=1, qs=s, k_pool=1, v_pool=1, num_layers=1, layer=0, capacity=4096, page_table=1,
                pts=32, cache_lens=1, q_start=1, q_len=1, out=1, os=s, batch=3, total=10, hq=32,
                hkv=8, head_dim=128, page_size=128, dtype=0, scale=0.088, dec=1, n_dec=1, pre=1,
                n_pre=2, max_q=8, max_kv=4096, split=0, ws=None, ws_bytes=0, err=None, stream=None)
    args.update(overrides)
    return list(args.values())


@pytest.mark.parametrize("bad, message", [
    (dict(q_start=None), "null pointer"),
    (dict(n_dec=0, n_pre=0), "at least one request"),
    (dict(pre=None), "null request list"),
    (dict(total=0), "total_tokens"),
    (dict(max_q=11), "max_query_len"),
    (dict(hq=30), "multiple of num_kv_heads"),
])
def test_packed_attention_rejects_bad_arguments(bad, message):
    lib = _lib.lib()
    rc = lib.hyt_paged_attention_packed(*_packed_args(**bad))
    assert rc == -1
    assert message in lib.hyt_last_error().decode()


def test_packed_scatter_rejects_bad_arguments():
    lib = _lib.lib()
    s = _lib.int64_array([0, 0, 0, 0])
    base = [1, 1, s, 1, 1, 1, 0, 1024, 1, 8, 1, 1, 1, 2, 5, 8, 128, 128, 0, None, None]
    args = list(base)
    args[12] = None  # token_request
    assert lib.hyt_kv_scatter_packed(*args) == -1
    args = list(base)
    args[14] = 0  # total_tokens
    assert lib.hyt_kv_scatter_packed(*args) == -1
    assert "total_tokens" in lib.hyt_last_error().decode()


def _planned_args(**overrides):
    """hyt_prefill_attention_planned arguments for a shape the prefill kernel takes (16-byte
    aligned fake pointers: nothing is dereferenced before the checks return)."""
    s = _lib.int64_array([0, 0, 0])
    args = dict(q=16, qs=s, k_pool=16, v_pool=16, num_layers=1, layer=0, capacity=4096,
                page_table=16, pts=32, cache_lens=16, out=16, os=s, batch=2, query_len=256,
                hq=32, hkv=8, head_dim=128, page_size=128, dtype=0, scale=0.088,
                items=16, num_items=4, num_splits=0, ws=None, ws_bytes=0, err=None, stream=None)
    args.update(overrides)
    return list(args.values())


@pytest.mark.parametrize("bad, code, message", [
    (dict(q=None), -1, "null pointer"),
    (dict(num_items=-1), -1, "bad plan"),
    (dict(items=None), -1, "bad plan"),
    (dict(num_splits=2), -4, "hyt_prefill_workspace_bytes"),
    (dict(num_splits=2, ws=16, ws_bytes=1024), -4, "hyt_prefill_workspace_bytes"),
    (dict(num_splits=2, ws=8, ws_bytes=1 << 30), -4, "not 16-byte aligned"),
    (dict(head_dim=64), -2, "prefill kernel needs"),
])
def test_planned_prefill_rejects_bad_arguments(bad, code, message):
    lib = _lib.lib()
    rc = lib.hyt_prefill_attention_planned(*_planned_args(**bad))
    assert rc == code
    assert message in lib.hyt_last_error().decode()


def test_planned_packed_attention_rejects_bad_plans():
    lib = _lib.lib()
    base = _packed_args()
    head, tail = base[:-2], base[-2:]  # ... workspace_bytes | error_word, stream
    assert lib.hyt_paged_attention_packed_planned(*head, None, 3, 0, None, 0, *tail) == -1
    assert "bad plan" in lib.hyt_last_error().decode()
    assert lib.hyt_paged_attention_packed_planned(*head, 16, 3, 4, None, 0, *tail) == -4
    assert "hyt_prefill_workspace_bytes" in lib.hyt_last_error().decode()


def test_fused_scatter_entry_rejects_null_rows():
    lib = _lib.lib()
    a = _attention_args()
    s6 = _lib.int64_array([0] * 6)
    # q, qs | k_new, v_new, new_strides | k_pool ... (the hyt_paged_attention arguments)
    rc = lib.hyt_paged_attention_scatter(a[0], a[1], None, 1, s6, *a[2:])
    assert rc == -1
    assert "null pointer" in lib.hyt_last_error().decode()


def test_prefill_plan_and_self_test_reject_bad_arguments():
    lib = _lib.lib()
    n = ctypes.c_int32(0)
    items = (ctypes.c_int32 * 16)()
    lens = (ctypes.c_int32 * 2)(10, 20)
    assert lib.hyt_prefill_plan(None, None, 2, 64, 32, 148, 8, 0.0, 0.0, items, 4, ctypes.byref(n)) == -1
    assert lib.hyt_prefill_plan(lens, None, 0, 64, 32, 148, 8, 0.0, 0.0, items, 4, ctypes.byref(n)) == -1
    assert lib.hyt_prefill_plan(lens, None, 2, 64, 32, 0, 8, 0.0, 0.0, items, 4, ctypes.byref(n)) == -1
    assert lib.hyt_wait_self_test(None, None, None) == -1
    assert "null" in lib.hyt_last_error().decode()


def _norm_rope_args(**overrides):
    """hyt_norm_rope_scatter arguments for a shape it takes (16-byte aligned fake pointers:
    nothing is dereferenced before the checks return)."""
    qkv = _lib.int64_array([4 * 48 * 128, 48 * 128, 128] * 3)
    outs = _lib.int64_array([32 * 4 * 128, 128, 32 * 128])
    args = dict(q=16, k=16, v=16, qkv=qkv, wq=16, wk=16, eps=1e-6, cos=16, sin=16, positions=4096,
                q_out=16, outs=outs, k_pool=16, v_pool=16, num_layers=1, layer=0, capacity=4096,
                page_table=16, pts=32, cache_lens=16, batch=2, query_len=4, hq=32, hkv=8,
                head_dim=128, page_size=128, dtype=0, err=None, stream=None)
    args.update(overrides)
    return list(args.values())


@pytest.mark.parametrize("bad, message", [
    (dict(q=24), "16-byte aligned"),        # 4-element (8-byte) aligned only
    (dict(wk=8), "16-byte aligned"),
    (dict(v_pool=40), "16-byte aligned"),
    (dict(qkv=_lib.int64_array([4 * 48 * 128, 48 * 128 + 4, 128] * 3)), "multiples of 16 bytes"),
    (dict(outs=_lib.int64_array([32 * 4 * 128, 132, 32 * 128])), "multiples of 16 bytes"),
    (dict(cos=8), "16-byte aligned"),
])
def test_fused_norm_rope_refuses_rows_off_16_byte_boundaries(bad, message):
    """The fused kernel moves 16 bytes per lane: a row that does not start on a 16-byte
    boundary is refused on the host instead of reaching the GPU."""
    lib = _lib.lib()
    rc = lib.hyt_norm_rope_scatter(*_norm_rope_args(**bad))
    assert rc == -1
    assert message in lib.hyt_last_error().decode()


def test_workspace_counter_layout_matches_the_library():
    """The Python managers zero only a workspace's counter bytes when a layout reaches past
    the known-zero prefix; their counter sizes must be the library's layout."""
    import torch

    from hayate_b200 import ops

    slot = 2 * (2 * 128 * 128 * 4 + 2 * 128 * 2 * 4)  # one prefill split slot's partials
    for n in (1, 63, 64, 65, 200):
        assert ops.prefill_workspace_bytes(n) == ops.prefill_counter_bytes(n) + n * slot
    # decode: 4 splits of 1024 keys, 4 rows (32 query heads / 8 KV heads, one query)
    for batch in (1, 7, 8, 9, 64, 100):
        units, splits, rows = batch * 8, 4, 4
        ml = -(-units * splits * rows * 2 * 4 // 256) * 256
        o = units * splits * rows * 128 * 4
        total = ops.attention_workspace_bytes(batch, 1, 32, 8, 128, 4096, torch.bfloat16, 1024)
        assert total - ml - o == ops.attention_counter_bytes(batch, 8)
