"""Tensor-level wrappers of the native kernels (device tensors in, device tensors out).

Each function checks devices, dtypes and layouts, hands raw pointers and
element strides to the C ABI and raises ``RuntimeError`` with the library's
message if the call is refused. All launches go on the current CUDA stream.
"""

from __future__ import annotations

import ctypes
import functools
import math

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.HYT_DTYPE_BF16, torch.float16: _lib.HYT_DTYPE_F16,
           torch.float32: _lib.HYT_DTYPE_F32}

KERNELS = ("auto", "decode", "prefill", "generic")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}; expected bf16, f16 or f32") from None


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("hayate_b200 kernels run on CUDA tensors only (no CPU fallback)")


def _stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _bht_strides(t: torch.Tensor, name: str) -> tuple[int, int, int]:
    if t.dim() != 4:
        raise ValueError(f"{name} must be [batch, heads, tokens, head_dim]")
    if t.stride(3) != 1 and t.size(3) > 1:
        raise ValueError(f"{name} must have a contiguous last dimension")
    return t.stride(0), t.stride(1), t.stride(2)


def _pool_geometry(k_pool: torch.Tensor, v_pool: torch.Tensor) -> tuple[int, int, int, int]:
    if k_pool.dim() != 5 or k_pool.size(1) != 1:
        raise ValueError("pools must be [num_layers, 1, num_kv_heads, capacity_tokens, head_dim]")
    if k_pool.shape != v_pool.shape or k_pool.dtype != v_pool.dtype:
        raise ValueError("K and V pools must have the same shape and dtype")
    if not (k_pool.is_contiguous() and v_pool.is_contiguous()):
        raise ValueError("pools must be contiguous")
    num_layers, _, heads, capacity, head_dim = k_pool.shape
    return num_layers, heads, capacity, head_dim


def _table_args(page_table: torch.Tensor, cache_lens: torch.Tensor, batch: int):
    if page_table.dtype != torch.int32 or cache_lens.dtype != torch.int32:
        raise TypeError("page_table and cache_lens must be int32")
    if page_table.dim() != 2 or page_table.size(0) != batch or page_table.stride(1) != 1:
        raise ValueError("page_table must be [batch, pages] with contiguous rows")
    if cache_lens.numel() != batch or not cache_lens.is_contiguous():
        raise ValueError("cache_lens must be a contiguous [batch] tensor")
    return page_table.stride(0)


def kv_scatter(k_new: torch.Tensor, v_new: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
               layer: int, page_table: torch.Tensor, cache_lens: torch.Tensor, page_size: int,
               error_word: torch.Tensor | None = None) -> None:
    """Kernel (a): write ``[B, H_kv, T, D]`` K/V into the pools at ``page_table`` slots."""
    _require_cuda(k_new, v_new, k_pool, v_pool, page_table, cache_lens)
    num_layers, heads, capacity, head_dim = _pool_geometry(k_pool, v_pool)
    if k_new.shape != v_new.shape or k_new.dtype != k_pool.dtype or v_new.dtype != k_pool.dtype:
        raise ValueError("k/v must share one shape and the pool dtype")
    batch, h, query_len, d = k_new.shape
    if h != heads or d != head_dim:
        raise ValueError("k/v heads and head_dim must match the pool")
    strides = _lib.int64_array(_bht_strides(k_new, "k") + _bht_strides(v_new, "v"))
    pts = _table_args(page_table, cache_lens, batch)
    rc = _lib.lib().hyt_kv_scatter(
        k_new.data_ptr(), v_new.data_ptr(), strides, k_pool.data_ptr(), v_pool.data_ptr(),
        num_layers, layer, capacity, page_table.data_ptr(), pts, cache_lens.data_ptr(), batch,
        query_len, heads, head_dim, page_size, dtype_code(k_pool.dtype), _ptr(error_word),
        _stream_ptr())
    _lib.check(rc, "hyt_kv_scatter")


def norm_rope_scatter(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_norm_weight: torch.Tensor,
                      k_norm_weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                      k_pool: torch.Tensor, v_pool: torch.Tensor, layer: int, page_table: torch.Tensor,
                      cache_lens: torch.Tensor, page_size: int, eps: float = 1e-6,
                      q_out: torch.Tensor | None = None,
                      error_word: torch.Tensor | None = None) -> torch.Tensor:
    """Fused QK-norm + RoPE + KV scatter: q/k/v are the projections ``[B, T, H, 128]``.

    Returns ``q`` normalised and rotated as ``[B, H_q, T, 128]`` (backed by ``[B, T, H_q, 128]``
    memory) and writes the normalised, rotated k and the raw v into the pools.
    """
    _require_cuda(q, k, v, q_norm_weight, k_norm_weight, cos, sin, k_pool, v_pool, page_table, cache_lens)
    num_layers, num_kv_heads, capacity, head_dim = _pool_geometry(k_pool, v_pool)
    if q.dim() != 4 or k.shape != v.shape or k.dim() != 4:
        raise ValueError("q, k, v must be [batch, tokens, heads, head_dim]")
    batch, query_len, num_q_heads, d = q.shape
    if d != head_dim or k.shape[2] != num_kv_heads or k.shape[:2] != q.shape[:2]:
        raise ValueError("q/k/v shapes do not match the pools")
    for t in (q, k, v, q_norm_weight, k_norm_weight):
        if t.dtype != k_pool.dtype:
            raise ValueError("q/k/v and the norm weights must have the pool dtype")
    if cos.dtype != torch.float32 or sin.dtype != torch.float32 or not (cos.is_contiguous() and sin.is_contiguous()):
        raise ValueError("cos/sin must be contiguous fp32 [positions, head_dim] tables")
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        if t.stride(3) != 1:
            raise ValueError(f"{name} must have a contiguous last dimension")
    if q_out is None:
        q_out = torch.empty((batch, query_len, num_q_heads, head_dim), dtype=q.dtype,
                            device=q.device).transpose(1, 2)
    strides = _lib.int64_array([q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1),
                                k.stride(2), v.stride(0), v.stride(1), v.stride(2)])
    out_strides = _lib.int64_array(_bht_strides(q_out, "q_out"))
    pts = _table_args(page_table, cache_lens, batch)
    rc = _lib.lib().hyt_norm_rope_scatter(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), strides, q_norm_weight.data_ptr(),
        k_norm_weight.data_ptr(), float(eps), cos.data_ptr(), sin.data_ptr(), cos.shape[0],
        q_out.data_ptr(), out_strides, k_pool.data_ptr(), v_pool.data_ptr(), num_layers, layer,
        capacity, page_table.data_ptr(), pts, cache_lens.data_ptr(), batch, query_len,
        num_q_heads, num_kv_heads, head_dim, page_size, dtype_code(q.dtype), _ptr(error_word),
        _stream_ptr())
    _lib.check(rc, "hyt_norm_rope_scatter")
    return q_out


@functools.lru_cache(maxsize=1024)
def attention_workspace_bytes(batch: int, query_len: int, num_q_heads: int, num_kv_heads: int,
                              head_dim: int, max_kv_len: int, dtype: torch.dtype,
                              split_tokens: int = 0) -> int:
    """Workspace bytes of a decode launch (``hyt_attention_workspace_bytes``; a pure function
    of its arguments, cached: every layer of every step asks)."""
    return int(_lib.lib().hyt_attention_workspace_bytes(batch, query_len, num_q_heads, num_kv_heads,
                                                        head_dim, max_kv_len, split_tokens,
                                                        dtype_code(dtype)))


def attention_counter_bytes(batch: int, num_kv_heads: int) -> int:
    """Leading bytes of a split-KV decode workspace that hold the per-(request, KV head)
    arrival counters: 4 bytes per unit, rounded up to 256 (the library's layout; pinned by
    tests/test_capi.py). The kernels need them zero at launch and leave them zero."""
    return -(-batch * num_kv_heads * 4 // 256) * 256


def prefill_counter_bytes(num_splits: int) -> int:
    """Leading bytes of a prefill-plan workspace that hold the split slots' counters (4 bytes
    per slot, rounded up to 256; the library's layout, pinned by tests/test_capi.py)."""
    return -(-num_splits * 4 // 256) * 256 if num_splits > 0 else 0


def new_workspace(nbytes: int, device) -> torch.Tensor:
    """A zeroed byte workspace (the kernels keep its counter area zero between calls)."""
    return torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=device)


def paged_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, layer: int,
                    page_table: torch.Tensor, cache_lens: torch.Tensor, page_size: int,
                    max_kv_len: int, scale: float | None = None, out: torch.Tensor | None = None,
                    workspace: torch.Tensor | None = None, error_word: torch.Tensor | None = None,
                    kernel: str = "auto", split_tokens: int = 0) -> torch.Tensor:
    """Causal GQA attention of ``q`` ``[B, H_q, T, D]`` over the paged pools.

    ``max_kv_len`` must be at least ``cache_lens[b] + T`` for every row.
    ``kernel`` pins one kernel instead of the library's choice.
    """
    if kernel not in KERNELS:
        raise ValueError(f"kernel must be one of {KERNELS}")
    _require_cuda(q, k_pool, v_pool, page_table, cache_lens)
    num_layers, num_kv_heads, capacity, head_dim = _pool_geometry(k_pool, v_pool)
    batch, num_q_heads, query_len, d = q.shape
    if d != head_dim or q.dtype != k_pool.dtype:
        raise ValueError("q must match the pool's head_dim and dtype")
    if out is None:
        # [B, T, H, D] memory viewed as [B, H, T, D]: the caller's transpose(1, 2) is then free
        out = torch.empty((batch, query_len, num_q_heads, head_dim), dtype=q.dtype,
                          device=q.device).transpose(1, 2)
    if out.shape != q.shape or out.dtype != q.dtype:
        raise ValueError("out must match q")
    qs = _lib.int64_array(_bht_strides(q, "q"))
    os_ = _lib.int64_array(_bht_strides(out, "out"))
    pts = _table_args(page_table, cache_lens, batch)
    scale = 1.0 / math.sqrt(head_dim) if scale is None else float(scale)
    lib = _lib.lib()
    common = (q.data_ptr(), qs, k_pool.data_ptr(), v_pool.data_ptr(), num_layers, layer, capacity,
              page_table.data_ptr(), pts, cache_lens.data_ptr(), out.data_ptr(), os_, batch,
              query_len, num_q_heads, num_kv_heads, head_dim, page_size, dtype_code(q.dtype), scale)
    stream = _stream_ptr()
    if kernel == "generic":
        rc = lib.hyt_generic_attention(*common, _ptr(error_word), stream)
    elif kernel == "prefill":
        rc = lib.hyt_prefill_attention(*common, max_kv_len, _ptr(error_word), stream)
    else:
        need = attention_workspace_bytes(batch, query_len, num_q_heads, num_kv_heads, head_dim,
                                         max_kv_len, q.dtype, split_tokens)
        if need and (workspace is None or workspace.numel() < need):
            raise RuntimeError(f"attention needs a zeroed workspace of {need} bytes")
        ws_ptr = _ptr(workspace) if need else None
        ws_bytes = workspace.numel() if (need and workspace is not None) else 0
        fn = lib.hyt_decode_attention if kernel == "decode" else lib.hyt_paged_attention
        rc = fn(*common, max_kv_len, split_tokens, ws_ptr, ws_bytes, _ptr(error_word), stream)
    _lib.check(rc, f"paged attention ({kernel})")
    return out


def paged_attention_scatter(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                            k_pool: torch.Tensor, v_pool: torch.Tensor, layer: int,
                            page_table: torch.Tensor, cache_lens: torch.Tensor, page_size: int,
                            max_kv_len: int, scale: float | None = None,
                            out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                            error_word: torch.Tensor | None = None,
                            split_tokens: int = 0) -> torch.Tensor:
    """``kv_scatter`` of the step's ``[B, H_kv, T, D]`` K/V, then ``paged_attention`` of
    ``q``: one launch when the decode kernel serves the step (``hyt_paged_attention_scatter``)."""
    _require_cuda(q, k_new, v_new, k_pool, v_pool, page_table, cache_lens)
    num_layers, num_kv_heads, capacity, head_dim = _pool_geometry(k_pool, v_pool)
    batch, num_q_heads, query_len, d = q.shape
    if d != head_dim or q.dtype != k_pool.dtype:
        raise ValueError("q must match the pool's head_dim and dtype")
    if k_new.shape != v_new.shape or k_new.dtype != k_pool.dtype or v_new.dtype != k_pool.dtype:
        raise ValueError("k/v must share one shape and the pool dtype")
    if tuple(k_new.shape) != (batch, num_kv_heads, query_len, head_dim):
        raise ValueError("k/v must be [batch, kv_heads, query_len, head_dim] of the pool")
    if out is None:
        out = torch.empty((batch, query_len, num_q_heads, head_dim), dtype=q.dtype,
                          device=q.device).transpose(1, 2)
    if out.shape != q.shape or out.dtype != q.dtype:
        raise ValueError("out must match q")
    qs = _lib.int64_array(_bht_strides(q, "q"))
    os_ = _lib.int64_array(_bht_strides(out, "out"))
    new_strides = _lib.int64_array(_bht_strides(k_new, "k") + _bht_strides(v_new, "v"))
    pts = _table_args(page_table, cache_lens, batch)
    scale = 1.0 / math.sqrt(head_dim) if scale is None else float(scale)
    need = attention_workspace_bytes(batch, query_len, num_q_heads, num_kv_heads, head_dim,
                                     max_kv_len, q.dtype, split_tokens)
    if need and (workspace is None or workspace.numel() < need):
        raise RuntimeError(f"attention needs a zeroed workspace of {need} bytes")
    rc = _lib.lib().hyt_paged_attention_scatter(
        q.data_ptr(), qs, k_new.data_ptr(), v_new.data_ptr(), new_strides, k_pool.data_ptr(),
        v_pool.data_ptr(), num_layers, layer, capacity, page_table.data_ptr(), pts,
        cache_lens.data_ptr(), out.data_ptr(), os_, batch, query_len, num_q_heads, num_kv_heads,
        head_dim, page_size, dtype_code(q.dtype), scale, max_kv_len, split_tokens,
        _ptr(workspace) if need else None, workspace.numel() if need else 0, _ptr(error_word),
        _stream_ptr())
    _lib.check(rc, "hyt_paged_attention_scatter")
    return out


# ---------------------------------------------------------------------------- packed batches
def _th_strides(t: torch.Tensor, name: str) -> tuple[int, int]:
    """Element strides {token, head} of a ``[1, H, N, D]`` packed tensor."""
    if t.dim() != 4 or t.shape[0] != 1:
        raise ValueError(f"{name} must be [1, heads, total_tokens, head_dim]")
    if t.stride(3) != 1 and t.size(3) > 1:
        raise ValueError(f"{name} must have a contiguous last dimension")
    return t.stride(2), t.stride(1)


def _int32_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise TypeError("packed-batch metadata must be contiguous int32 tensors")


def kv_scatter_packed(k_new: torch.Tensor, v_new: torch.Tensor, k_pool: torch.Tensor,
                      v_pool: torch.Tensor, layer: int, page_table: torch.Tensor,
                      cache_lens: torch.Tensor, q_start: torch.Tensor, token_request: torch.Tensor,
                      page_size: int, error_word: torch.Tensor | None = None) -> None:
    """Kernel (a) on a packed batch: ``[1, H_kv, N, D]`` new K/V, token i of request
    ``token_request[i]`` at position ``cache_lens[b] + i - q_start[b]``."""
    _require_cuda(k_new, v_new, k_pool, v_pool, page_table, cache_lens, q_start, token_request)
    _int32_cuda(q_start, token_request)
    num_layers, heads, capacity, head_dim = _pool_geometry(k_pool, v_pool)
    if k_new.shape != v_new.shape or k_new.dtype != k_pool.dtype or v_new.dtype != k_pool.dtype:
        raise ValueError("k/v must share one shape and the pool dtype")
    _, h, total, d = k_new.shape
    if h != heads or d != head_dim or token_request.numel() != total:
        raise ValueError("k/v heads, head_dim and token count must match the pool and metadata")
    batch = cache_lens.numel()
    strides = _lib.int64_array(_th_strides(k_new, "k") + _th_strides(v_new, "v"))
    pts = _table_args(page_table, cache_lens, batch)
    rc = _lib.lib().hyt_kv_scatter_packed(
        k_new.data_ptr(), v_new.data_ptr(), strides, k_pool.data_ptr(), v_pool.data_ptr(),
        num_layers, layer, capacity, page_table.data_ptr(), pts, cache_lens.data_ptr(),
        q_start.data_ptr(), token_request.data_ptr(), batch, total, heads, head_dim, page_size,
        dtype_code(k_pool.dtype), _ptr(error_word), _stream_ptr())
    _lib.check(rc, "hyt_kv_scatter_packed")


def norm_rope_scatter_packed(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                             q_norm_weight: torch.Tensor, k_norm_weight: torch.Tensor,
                             cos: torch.Tensor, sin: torch.Tensor, k_pool: torch.Tensor,
                             v_pool: torch.Tensor, layer: int, page_table: torch.Tensor,
                             cache_lens: torch.Tensor, q_start: torch.Tensor,
                             token_request: torch.Tensor, page_size: int, eps: float = 1e-6,
                             error_word: torch.Tensor | None = None) -> torch.Tensor:
    """Fused QK-norm + RoPE + scatter on a packed batch: q/k/v are the projections as
    ``[1, N, H, 128]``; returns the rotated q as ``[1, H_q, N, 128]`` (backed by
    ``[1, N, H_q, 128]`` memory)."""
    _require_cuda(q, k, v, q_norm_weight, k_norm_weight, cos, sin, k_pool, v_pool, page_table,
                  cache_lens, q_start, token_request)
    _int32_cuda(q_start, token_request)
    num_layers, num_kv_heads, capacity, head_dim = _pool_geometry(k_pool, v_pool)
    if q.dim() != 4 or q.shape[0] != 1 or k.shape != v.shape or k.shape[:2] != q.shape[:2]:
        raise ValueError("q, k, v must be [1, total_tokens, heads, head_dim]")
    _, total, num_q_heads, d = q.shape
    if d != head_dim or k.shape[2] != num_kv_heads or token_request.numel() != total:
        raise ValueError("q/k/v shapes do not match the pools and metadata")
    for t in (q, k, v, q_norm_weight, k_norm_weight):
        if t.dtype != k_pool.dtype:
            raise ValueError("q/k/v and the norm weights must have the pool dtype")
    if cos.dtype != torch.float32 or sin.dtype != torch.float32 or not (cos.is_contiguous() and sin.is_contiguous()):
        raise ValueError("cos/sin must be contiguous fp32 [positions, head_dim] tables")
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        if t.stride(3) != 1:
            raise ValueError(f"{name} must have a contiguous last dimension")
    q_out = torch.empty((1, total, num_q_heads, head_dim), dtype=q.dtype, device=q.device).transpose(1, 2)
    strides = _lib.int64_array([q.stride(1), q.stride(2), k.stride(1), k.stride(2), v.stride(1), v.stride(2)])
    out_strides = _lib.int64_array(_th_strides(q_out, "q_out"))
    batch = cache_lens.numel()
    pts = _table_args(page_table, cache_lens, batch)
    rc = _lib.lib().hyt_norm_rope_scatter_packed(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), strides, q_norm_weight.data_ptr(),
        k_norm_weight.data_ptr(), float(eps), cos.data_ptr(), sin.data_ptr(), cos.shape[0],
        q_out.data_ptr(), out_strides, k_pool.data_ptr(), v_pool.data_ptr(), num_layers, layer,
        capacity, page_table.data_ptr(), pts, cache_lens.data_ptr(), q_start.data_ptr(),
        token_request.data_ptr(), batch, total, num_q_heads, num_kv_heads, head_dim, page_size,
        dtype_code(q.dtype), _ptr(error_word), _stream_ptr())
    _lib.check(rc, "hyt_norm_rope_scatter_packed")
    return q_out


def paged_attention_packed(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, layer: int,
                           page_table: torch.Tensor, cache_lens: torch.Tensor, q_start: torch.Tensor,
                           q_len: torch.Tensor, decode_ids: torch.Tensor, prefill_ids: torch.Tensor,
                           page_size: int, max_query_len: int, max_kv_len: int,
                           scale: float | None = None, out: torch.Tensor | None = None,
                           workspace: torch.Tensor | None = None,
                           error_word: torch.Tensor | None = None, split_tokens: int = 0,
                           plan_items: torch.Tensor | None = None, plan_splits: int = 0,
                           plan_workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Causal GQA attention of a packed batch ``q`` ``[1, H_q, N, D]``: the requests in
    ``decode_ids`` (one query each) on the decode kernel, those in ``prefill_ids`` on the
    prefill kernel, in one call. ``plan_items`` (int32 ``[n, 4]`` CUDA, from
    ``prefill_plan`` over the prefill requests in ``prefill_ids`` order) schedules the
    prefill launch."""
    _require_cuda(q, k_pool, v_pool, page_table, cache_lens, q_start, q_len, decode_ids, prefill_ids)
    _int32_cuda(q_start, q_len, decode_ids, prefill_ids)
    num_layers, num_kv_heads, capacity, head_dim = _pool_geometry(k_pool, v_pool)
    _, num_q_heads, total, d = q.shape
    if d != head_dim or q.dtype != k_pool.dtype:
        raise ValueError("q must match the pool's head_dim and dtype")
    if out is None:
        out = torch.empty((1, total, num_q_heads, head_dim), dtype=q.dtype, device=q.device).transpose(1, 2)
    if out.shape != q.shape or out.dtype != q.dtype:
        raise ValueError("out must match q")
    qs = _lib.int64_array(_th_strides(q, "q"))
    os_ = _lib.int64_array(_th_strides(out, "out"))
    batch = cache_lens.numel()
    pts = _table_args(page_table, cache_lens, batch)
    n_dec, n_pre = decode_ids.numel(), prefill_ids.numel()
    scale = 1.0 / math.sqrt(head_dim) if scale is None else float(scale)
    need = attention_workspace_bytes(n_dec, 1, num_q_heads, num_kv_heads, head_dim, max_kv_len,
                                     q.dtype, split_tokens) if n_dec else 0
    if need and (workspace is None or workspace.numel() < need):
        raise RuntimeError(f"attention needs a zeroed workspace of {need} bytes")
    common = (q.data_ptr(), qs, k_pool.data_ptr(), v_pool.data_ptr(), num_layers, layer, capacity,
              page_table.data_ptr(), pts, cache_lens.data_ptr(), q_start.data_ptr(), q_len.data_ptr(),
              out.data_ptr(), os_, batch, total, num_q_heads, num_kv_heads, head_dim, page_size,
              dtype_code(q.dtype), scale, decode_ids.data_ptr() if n_dec else None, n_dec,
              prefill_ids.data_ptr() if n_pre else None, n_pre, max_query_len, max_kv_len,
              split_tokens, _ptr(workspace) if need else None, workspace.numel() if need else 0)
    if plan_items is None:
        rc = _lib.lib().hyt_paged_attention_packed(*common, _ptr(error_word), _stream_ptr())
        _lib.check(rc, "hyt_paged_attention_packed")
        return out
    pneed = _check_plan(plan_items, plan_splits, plan_workspace)
    rc = _lib.lib().hyt_paged_attention_packed_planned(
        *common, plan_items.data_ptr(), plan_items.shape[0], plan_splits,
        _ptr(plan_workspace) if pneed else None, plan_workspace.numel() if pneed else 0,
        _ptr(error_word), _stream_ptr())
    _lib.check(rc, "hyt_paged_attention_packed_planned")
    return out


def read_device_errors(error_word: torch.Tensor) -> list[str]:
    """Decode (and synchronise on) a device error word; empty if no kernel refused anything."""
    value = int(error_word.item())
    return [msg for bit, msg in _lib.DEVICE_ERRORS.items() if value & bit]


def wait_self_test(error_word: torch.Tensor) -> tuple[int, int]:
    """Run the bounded-wait self-test (``hyt_wait_self_test``) on the current stream.

    A wait on an mbarrier that nothing signals gives up after its 1 s limit and ORs the
    wait-timeout bit into ``error_word``; a second wait of the same CTA then returns at
    once. Returns both waits' durations in nanoseconds (synchronises).
    """
    _require_cuda(error_word)
    if error_word.dtype != torch.int32 or error_word.numel() < 1:
        raise ValueError("error_word must be a CUDA int32 tensor")
    elapsed = torch.zeros(2, dtype=torch.int64, device=error_word.device)
    rc = _lib.lib().hyt_wait_self_test(error_word.data_ptr(), elapsed.data_ptr(), _stream_ptr())
    _lib.check(rc, "hyt_wait_self_test")
    first, second = elapsed.tolist()
    return first, second


def read_probe(buf: torch.Tensor, sink: torch.Tensor) -> None:
    """Launch the plain streaming-read kernel (``hyt_read_probe``) over ``buf``'s bytes on the
    current stream: the HBM read ceiling the decode kernel is compared with (measurement only).
    ``sink`` is a CUDA int32 tensor with one element per CTA (its length sets the grid)."""
    _require_cuda(buf)
    _require_cuda(sink)
    if sink.dtype != torch.int32 or not sink.is_contiguous() or not buf.is_contiguous():
        raise ValueError("buf must be contiguous and sink a contiguous int32 tensor")
    nbytes = buf.numel() * buf.element_size()
    rc = _lib.lib().hyt_read_probe(buf.data_ptr(), nbytes, sink.data_ptr(), sink.numel(), _stream_ptr())
    _lib.check(rc, "hyt_read_probe")


# ---------------------------------------------------------------------------- prefill schedule
def prefill_plan(cache_lens, query_len: int, num_q_heads: int, num_sms: int, max_splits: int = 128,
                 q_lens=None, item_overhead: float = 0.0, merge_cost: float = 0.0):
    """Host-side schedule for the prefill kernel (``hyt_prefill_plan``).

    ``cache_lens`` / ``q_lens`` are host sequences (one entry per request of the launch);
    ``item_overhead`` / ``merge_cost`` override the cost model's constants (key tiles;
    0 keeps the library's defaults). Returns ``(items, num_splits)``: ``items`` an int32 ``[n, 4]`` array for
    ``prefill_attention_planned``, or ``None`` when the default grid is at least as good.
    """
    import numpy as np

    lens = np.ascontiguousarray(np.asarray(cache_lens, dtype=np.int32))
    ql = None if q_lens is None else np.ascontiguousarray(np.asarray(q_lens, dtype=np.int32))
    batch = lens.size
    qmax = int(ql.max()) if ql is not None else int(query_len)
    tiles = sum(-(-int(n) // 128) for n in ql) if ql is not None else batch * -(-qmax // 128)
    max_items = tiles * (num_q_heads // 2) + max_splits
    items = np.zeros((max(max_items, 1), 4), dtype=np.int32)
    splits = ctypes.c_int32(0)
    n = _lib.lib().hyt_prefill_plan(lens.ctypes.data, None if ql is None else ql.ctypes.data, batch,
                                    qmax, num_q_heads, num_sms, max_splits, item_overhead, merge_cost,
                                    items.ctypes.data, max_items, ctypes.byref(splits))
    if n < 0:
        _lib.check(n, "hyt_prefill_plan")
    return (items[:n].copy(), int(splits.value)) if n > 0 else (None, 0)


def prefill_workspace_bytes(num_splits: int) -> int:
    return int(_lib.lib().hyt_prefill_workspace_bytes(num_splits))


def _check_plan(items: torch.Tensor, num_splits: int, workspace: torch.Tensor | None) -> int:
    """Validate a plan's device items and split workspace; returns the workspace bytes needed."""
    _require_cuda(items)
    if items.dtype != torch.int32 or items.dim() != 2 or items.shape[1] != 4 or not items.is_contiguous():
        raise ValueError("plan items must be a contiguous int32 [n, 4] CUDA tensor")
    need = prefill_workspace_bytes(num_splits)
    if need and (workspace is None or workspace.numel() < need):
        raise RuntimeError(f"the plan needs a zeroed workspace of {need} bytes")
    return need


def prefill_attention_planned(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, layer: int,
                              page_table: torch.Tensor, cache_lens: torch.Tensor, page_size: int,
                              items: torch.Tensor | None, num_splits: int,
                              workspace: torch.Tensor | None = None, scale: float | None = None,
                              out: torch.Tensor | None = None,
                              error_word: torch.Tensor | None = None) -> torch.Tensor:
    """The tcgen05 prefill kernel launched on a plan from ``prefill_plan`` (``items`` an
    int32 ``[n, 4]`` CUDA tensor; ``None`` runs the default grid)."""
    _require_cuda(q, k_pool, v_pool, page_table, cache_lens)
    num_layers, num_kv_heads, capacity, head_dim = _pool_geometry(k_pool, v_pool)
    batch, num_q_heads, query_len, d = q.shape
    if d != head_dim or q.dtype != k_pool.dtype:
        raise ValueError("q must match the pool's head_dim and dtype")
    if out is None:
        out = torch.empty((batch, query_len, num_q_heads, head_dim), dtype=q.dtype,
                          device=q.device).transpose(1, 2)
    if out.shape != q.shape or out.dtype != q.dtype:
        raise ValueError("out must match q")
    n_items = 0 if items is None else items.shape[0]
    need = _check_plan(items, num_splits, workspace) if n_items else 0
    qs = _lib.int64_array(_bht_strides(q, "q"))
    os_ = _lib.int64_array(_bht_strides(out, "out"))
    pts = _table_args(page_table, cache_lens, batch)
    scale = 1.0 / math.sqrt(head_dim) if scale is None else float(scale)
    rc = _lib.lib().hyt_prefill_attention_planned(
        q.data_ptr(), qs, k_pool.data_ptr(), v_pool.data_ptr(), num_layers, layer, capacity,
        page_table.data_ptr(), pts, cache_lens.data_ptr(), out.data_ptr(), os_, batch, query_len,
        num_q_heads, num_kv_heads, head_dim, page_size, dtype_code(q.dtype), scale,
        items.data_ptr() if n_items else None, n_items, num_splits if n_items else 0,
        _ptr(workspace) if need else None, workspace.numel() if need else 0, _ptr(error_word),
        _stream_ptr())
    _lib.check(rc, "hyt_prefill_attention_planned")
    return out
