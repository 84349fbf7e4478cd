"""Drop-in paged KV pool for hayate, backed by the hayate_b200 CUDA kernels.

Same public surface as ``hayate/engine/paged_cache.py``:

* ``PagedCacheHandle`` (``:23-30``), ``PagedKVCacheManager`` (``:74-315``) with
  ``allocate``/``reserve``/``allocate_for_request``/``import_cache``/``truncate``/
  ``snapshot``/``release``/``begin_batch``/``commit_batch`` and the same
  arguments, free-list order and exceptions (``ValueError``, ``RuntimeError``,
  ``MemoryError``);
* ``begin_batch`` returns a ``PagedKVBatch`` exposing ``write_layer(layer, k, v)``,
  ``attend_layer(q, layer)``, ``cache_lens`` (int64, read by the model to place
  RoPE positions), ``page_table`` and ``page_size`` (``:33-71``), plus
  ``prepare_layer`` (QK-norm + RoPE + ``write_layer`` fused in one launch).

What changes underneath:

* ``write_layer`` is one launch of the scatter kernel and ``attend_layer`` one
  launch of the decode, prefill or CUDA-core attention kernel. There is no
  block mask and no ``physical_to_logical`` table: the kernels walk the page
  table and apply the causal rule ``key <= cache_len + t`` themselves.
* Page tables persist per request slot on the device: a step uploads only the
  rows whose pages changed (usually none while decoding inside a page), its
  lengths and slot ids in one small copy, and gathers its ``[B, W]`` int32 table
  (``W`` = pages of the longest request) on the device, instead of one copy per
  request plus a block mask.
* Pages carry reference counts, so ``share`` can alias a prefix's physical
  pages into another request (prefix-cache page sharing). ``release`` and
  ``truncate`` decrement; a page returns to the free list at zero. A write that
  would land in a page someone else still holds copies that page first.
* Pools start zeroed (the reference uses ``torch.empty``): tiles that straddle
  a request's last token read finite bytes, so masked keys contribute exactly 0.
* ``attend_layer`` returns ``[B, H_q, T, D]`` backed by ``[B, T, H_q, D]``
  memory, so the attention module's ``transpose(1, 2).reshape(...)`` is free.

Pools may live on the CPU for the bookkeeping API (allocation, import,
snapshot); ``write_layer``/``attend_layer`` run on CUDA only and raise otherwise.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np
import torch

from . import ops
from .cache import KVSnapshot

MIN_KV_PAGE_SIZE = 128  # hayate/engine/constants.py:27 (FlexAttention block size floor)


@dataclass
class PagedCacheHandle:
    """One request's physical KV pages and logical cache length."""

    slot: int
    pages: list[int] = field(default_factory=list)
    length: int = 0
    released: bool = False
    aliased: bool = False  # some page may be shared with another request (set by share)


class _MetaUploader:
    """Asynchronous host-to-device upload of a step's packed metadata.

    A small ring of pinned host buffers, each guarded by the CUDA event of its
    last copy, so ``begin_batch`` never blocks on the GPU queue.
    """

    def __init__(self, device: torch.device, slots: int = 4):
        self.device = device
        self.buffers: list[torch.Tensor | None] = [None] * slots
        self.events: list[torch.cuda.Event | None] = [None] * slots
        self.index = 0

    def upload(self, host: np.ndarray) -> torch.Tensor:
        if self.device.type != "cuda":
            return torch.from_numpy(host.copy()).to(self.device)
        i = self.index
        self.index = (i + 1) % len(self.buffers)
        if self.events[i] is not None:
            self.events[i].synchronize()
        buf = self.buffers[i]
        if buf is None or buf.numel() < host.size:
            buf = torch.empty(max(host.size, 4096), dtype=torch.int32, pin_memory=True)
            self.buffers[i] = buf
        staged = buf[: host.size]
        staged.numpy()[:] = host
        dev = torch.empty(host.size, dtype=torch.int32, device=self.device)
        dev.copy_(staged, non_blocking=True)
        event = torch.cuda.Event()
        event.record()
        self.events[i] = event
        return dev


class _SlotPageTable:
    """Page-table rows kept per request slot, on the host and on the device.

    Row ``s`` lists slot ``s``'s physical pages in logical order (-1 past the end).
    The manager updates a row whenever that request's pages change; ``flush`` uploads
    only the rows changed since the previous step (one packed copy plus a device
    row copy), and ``gather`` builds a step's ``[B, W]`` table on the device from the
    batch's slots. A decode step that crosses no page boundary uploads no row at all.
    """

    def __init__(self, max_requests: int, device: torch.device, width: int = 64):
        self.device = device
        self.host = np.full((max_requests, width), -1, dtype=np.int32)
        self.count = np.zeros(max_requests, dtype=np.int64)
        self.dirty: set[int] = set()
        self.dev = torch.full((max_requests, width), -1, dtype=torch.int32, device=device)
        self.uploader = _MetaUploader(device)

    def _ensure_width(self, needed: int) -> None:
        width = self.host.shape[1]
        if needed <= width:
            return
        grown = max(needed, 2 * width)
        host = np.full((self.host.shape[0], grown), -1, dtype=np.int32)
        host[:, :width] = self.host
        self.host = host
        self.dev = torch.full((self.host.shape[0], grown), -1, dtype=torch.int32, device=self.device)
        self.dirty.update(int(s) for s in np.nonzero(self.count)[0])

    def set_row(self, slot: int, pages: Sequence[int]) -> None:
        n = len(pages)
        self._ensure_width(n)
        old = int(self.count[slot])
        if n:
            self.host[slot, :n] = pages
        if old > n:
            self.host[slot, n:old] = -1
        self.count[slot] = n
        self.dirty.add(slot)

    def append(self, slot: int, pages: Sequence[int]) -> None:
        start = int(self.count[slot])
        end = start + len(pages)
        self._ensure_width(end)
        self.host[slot, start:end] = pages
        self.count[slot] = end
        self.dirty.add(slot)

    def set_entry(self, slot: int, index: int, page: int) -> None:
        self.host[slot, index] = page
        self.dirty.add(slot)

    def flush(self) -> None:
        if not self.dirty:
            return
        rows = np.fromiter(sorted(self.dirty), dtype=np.int32, count=len(self.dirty))
        self.dirty.clear()
        width = self.host.shape[1]
        packed = np.concatenate([rows, self.host[rows].reshape(-1)])
        dev = self.uploader.upload(packed)
        n = len(rows)
        self.dev.index_copy_(0, dev[:n].long(), dev[n:].view(n, width))

    def gather(self, slots: torch.Tensor, width: int) -> torch.Tensor:
        return self.dev[:, :width].index_select(0, slots)


@dataclass
class PackedLayout:
    """Where each request's new tokens sit on a packed batch's shared token axis."""

    query_lens: list[int]      # tokens of each request this step
    total_tokens: int
    q_start: torch.Tensor      # [B] int32: first token row of each request
    q_len: torch.Tensor        # [B] int32
    token_request: torch.Tensor  # [total_tokens] int32: request of each token row
    decode_ids: torch.Tensor   # requests with one token (split-KV decode kernel)
    prefill_ids: torch.Tensor  # the others (tcgen05 prefill kernel)


class PagedKVBatch:
    """Per-step metadata shared by every layer of one forward pass.

    A packed batch (``begin_batch`` given one query length per request) puts every
    request's new tokens on one token axis, in batch order: tensors are ``[1, H, N, D]``
    (``N`` = total new tokens) and ``layout`` says which rows belong to which request.
    """

    __slots__ = ("k_cache", "v_cache", "page_table", "cache_lens", "page_size", "query_len",
                 "max_kv_len", "cache_lens_i32", "layout", "workspace", "_manager", "_meta",
                 "_host_lens", "_plans")

    def __init__(self, manager, page_table, cache_lens, cache_lens_i32, query_len, max_kv_len, meta,
                 layout: PackedLayout | None = None, host_lens=None):
        self.k_cache = manager.k_cache
        self.v_cache = manager.v_cache
        self.page_table = page_table
        self.cache_lens = cache_lens
        self.cache_lens_i32 = cache_lens_i32
        self.page_size = manager.page_size
        self.query_len = query_len
        self.max_kv_len = max_kv_len
        self.layout = layout
        self.workspace = None  # a batch with a fixed workspace (graph replays) sets its own
        self._manager = manager
        self._meta = meta  # keeps the uploaded buffer alive while kernels read it
        self._host_lens = host_lens  # cache lengths on the host (the prefill schedule's input)
        self._plans = {}             # num_q_heads -> (plan items on the device or None, splits)

    def write_layer(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Scatter the step's new K/V ``[B, H_kv, T, D]`` into this layer's pages."""
        if self.layout is not None:
            self._write_packed(layer_idx, k, v)
            return
        if k.shape[2] != self.query_len or v.shape != k.shape:
            raise ValueError("k and v must be [batch, kv_heads, query_len, head_dim]")
        if k.stride(-1) != 1:
            k = k.contiguous()
        if v.stride(-1) != 1:
            v = v.contiguous()
        ops.kv_scatter(k, v, self.k_cache, self.v_cache, layer_idx, self.page_table,
                       self.cache_lens_i32, self.page_size, error_word=self._manager.error_word)

    def prepare_layer(self, layer_idx: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      q_norm_weight: torch.Tensor, k_norm_weight: torch.Tensor,
                      cos: torch.Tensor, sin: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
        """QK-norm, RoPE and ``write_layer`` fused in one launch.

        ``q``/``k``/``v`` are the projections as ``[B, T, H, D]`` (before the transpose of
        ``hayate/model/attention.py:66-68``); the K/V written to the pages are those the
        unfused path (norm -> transpose -> RoPE -> ``write_layer``) writes. Returns the
        rotated ``q`` as ``[B, H_q, T, D]``, ready for ``attend_layer``.
        """
        if self.layout is not None:
            lay = self.layout
            if q.shape[0] != 1 or q.shape[1] != lay.total_tokens:
                raise ValueError("a packed batch's q/k/v are [1, total_tokens, heads, head_dim]")
            return ops.norm_rope_scatter_packed(
                q, k, v, q_norm_weight, k_norm_weight, cos, sin, self.k_cache, self.v_cache,
                layer_idx, self.page_table, self.cache_lens_i32, lay.q_start, lay.token_request,
                self.page_size, eps=eps, error_word=self._manager.error_word)
        if q.shape[1] != self.query_len:
            raise ValueError("q/k/v must carry query_len tokens")
        return ops.norm_rope_scatter(q, k, v, q_norm_weight, k_norm_weight, cos, sin, self.k_cache,
                                     self.v_cache, layer_idx, self.page_table, self.cache_lens_i32,
                                     self.page_size, eps=eps, error_word=self._manager.error_word)

    def attend_layer(self, q: torch.Tensor, layer_idx: int) -> torch.Tensor:
        """Causal GQA attention of ``q`` ``[B, H_q, T, D]`` over this layer's paged K/V."""
        if q.stride(-1) != 1:
            q = q.contiguous()
        manager = self._manager
        if self.layout is not None:
            lay = self.layout
            if q.shape[0] != 1 or q.shape[2] != lay.total_tokens:
                raise ValueError("a packed batch's q is [1, H_q, total_tokens, head_dim]")
            n_dec = lay.decode_ids.numel()
            workspace = self.workspace
            if workspace is None and n_dec:
                workspace = manager.workspace_for(n_dec, 1, q.shape[1], self.max_kv_len)
            planned = self.prefill_schedule(q)
            items, splits = planned if planned is not None else (None, 0)
            return ops.paged_attention_packed(
                q, self.k_cache, self.v_cache, layer_idx, self.page_table, self.cache_lens_i32,
                lay.q_start, lay.q_len, lay.decode_ids, lay.prefill_ids, self.page_size,
                self.query_len, self.max_kv_len, workspace=workspace, error_word=manager.error_word,
                split_tokens=manager.split_tokens, plan_items=items, plan_splits=splits,
                plan_workspace=manager.prefill_workspace(splits) if items is not None else None)
        planned = self.prefill_schedule(q)
        if planned is not None:
            items, splits = planned
            return ops.prefill_attention_planned(
                q, self.k_cache, self.v_cache, layer_idx, self.page_table, self.cache_lens_i32,
                self.page_size, items, splits, workspace=manager.prefill_workspace(splits),
                error_word=manager.error_word)
        workspace = manager.workspace_for(q.shape[0], self.query_len, q.shape[1], self.max_kv_len)
        return ops.paged_attention(q, self.k_cache, self.v_cache, layer_idx, self.page_table,
                                   self.cache_lens_i32, self.page_size, self.max_kv_len,
                                   workspace=workspace, error_word=manager.error_word,
                                   kernel=manager.kernel, split_tokens=manager.split_tokens)

    def write_attend_layer(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor,
                           q: torch.Tensor) -> torch.Tensor:
        """``write_layer(layer_idx, k, v)`` then ``attend_layer(q, layer_idx)``, the pair
        hayate's attention layer calls back to back (``hayate/model/attention.py``), with the
        same pool bytes and rows. A decode step runs as one launch: the decode kernel writes
        the new K/V rows itself before reading them."""
        manager = self._manager
        decode_step = (q.dtype in (torch.bfloat16, torch.float16) and q.shape[-1] == 128
                       and self.page_size % 64 == 0
                       and (q.shape[1] // manager.num_kv_heads) * self.query_len <= 16)
        if self.layout is not None or manager.kernel != "auto" or not decode_step:
            self.write_layer(layer_idx, k, v)  # the two kernels in turn (prefill: its schedule)
            return self.attend_layer(q, layer_idx)
        if k.shape[2] != self.query_len or v.shape != k.shape:
            raise ValueError("k and v must be [batch, kv_heads, query_len, head_dim]")
        if k.stride(-1) != 1:
            k = k.contiguous()
        if v.stride(-1) != 1:
            v = v.contiguous()
        if q.stride(-1) != 1:
            q = q.contiguous()
        workspace = manager.workspace_for(q.shape[0], self.query_len, q.shape[1], self.max_kv_len)
        return ops.paged_attention_scatter(q, k, v, self.k_cache, self.v_cache, layer_idx,
                                           self.page_table, self.cache_lens_i32, self.page_size,
                                           self.max_kv_len, workspace=workspace,
                                           error_word=manager.error_word,
                                           split_tokens=manager.split_tokens)

    def prefill_schedule(self, q: torch.Tensor):
        """(items, splits) for a planned prefill launch of this batch, or None for the
        library's own dispatch. The plan (``ops.prefill_plan``: longest items first, the
        heaviest cut in two) is made on the host once per batch and head count and reused
        by every layer."""
        manager = self._manager
        if (manager.kernel != "auto" or not manager.prefill_plan or self._host_lens is None
                or q.dtype not in (torch.bfloat16, torch.float16) or q.shape[3] != 128
                or self.page_size % 128 or q.device.type != "cuda"):
            return None
        heads = q.shape[1]
        group = heads // manager.num_kv_heads
        if q.data_ptr() % 16 or any(st % 8 for st in q.stride()[:3]) or group % 2:
            return None
        lay = self.layout
        if lay is None:
            if group * self.query_len <= 16:  # the decode kernel's shapes
                return None
            lens, q_lens = self._host_lens, None
        else:  # the packed batch's prefill requests, in prefill_ids order
            ids = [i for i, t in enumerate(lay.query_lens) if t > 1]
            if not ids:
                return None
            lens = [self._host_lens[i] for i in ids]
            q_lens = [lay.query_lens[i] for i in ids]
        if heads not in self._plans:
            items, splits = ops.prefill_plan(lens, self.query_len, heads, manager.num_sms,
                                             manager.prefill_max_splits, q_lens=q_lens)
            if items is not None:  # one pinned asynchronous upload per batch
                items = manager._uploader.upload(items.reshape(-1)).view(-1, 4)
            self._plans[heads] = (items, splits)
        items, splits = self._plans[heads]
        return None if items is None else (items, splits)

    def _write_packed(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
        lay = self.layout
        if k.shape[0] != 1 or k.shape[2] != lay.total_tokens or v.shape != k.shape:
            raise ValueError("a packed batch's k and v are [1, kv_heads, total_tokens, head_dim]")
        if k.stride(-1) != 1:
            k = k.contiguous()
        if v.stride(-1) != 1:
            v = v.contiguous()
        ops.kv_scatter_packed(k, v, self.k_cache, self.v_cache, layer_idx, self.page_table,
                              self.cache_lens_i32, lay.q_start, lay.token_request, self.page_size,
                              error_word=self._manager.error_word)


class StaticDecodeBatch:
    """A packed one-token-per-request batch of fixed size whose device buffers never move,
    for capturing a decode step in a CUDA graph and replaying it every tick.

    ``update(handles)`` (at most ``size`` requests, each with cache length + 1 <=
    ``max_kv_len``) does the step's page bookkeeping (``begin_batch``'s) and copies the
    lengths, slots and page rows into the buffers on the current stream. Rows past the real
    requests are padding: length 0 on the manager's scratch page, which nothing else uses,
    so their (discarded) writes and reads stay inside the pool.
    """

    def __init__(self, manager: "PagedKVCacheManager", size: int, max_kv_len: int, num_q_heads: int):
        if size < 1 or max_kv_len < 1 or max_kv_len > manager.capacity_tokens:
            raise ValueError("static batch size and max_kv_len must be positive and within the pool")
        device = manager.device
        self.size, self.max_kv_len = size, max_kv_len
        self.width = -(-max_kv_len // manager.page_size)
        manager._ensure_scratch_page()
        manager._rows._ensure_width(self.width)
        self.meta = torch.zeros(4 * size, dtype=torch.int32, device=device)  # [lens64 | lens32 | slots]
        self.table = torch.full((size, self.width), -1, dtype=torch.int32, device=device)
        rows = torch.arange(size, dtype=torch.int32, device=device)
        layout = PackedLayout(query_lens=[1] * size, total_tokens=size, q_start=rows,
                              q_len=torch.ones(size, dtype=torch.int32, device=device),
                              token_request=rows, decode_ids=rows, prefill_ids=rows[:0])
        self.batch = PagedKVBatch(manager, self.table, self.meta[: 2 * size].view(torch.int64),
                                  self.meta[2 * size: 3 * size], 1, max_kv_len, (self.meta, self.table),
                                  layout)
        need = ops.attention_workspace_bytes(size, 1, num_q_heads, manager.num_kv_heads,
                                             manager.head_dim, max_kv_len, manager.k_cache.dtype,
                                             manager.split_tokens)
        self.batch.workspace = ops.new_workspace(need, device) if need else None
        pin = device.type == "cuda"
        self._staging = [torch.empty(4 * size, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self._events: list = [None, None]
        self._flip = 0
        self._manager = manager

    def update(self, handles: Sequence[PagedCacheHandle]) -> None:
        m = self._manager
        n = len(handles)
        if n > self.size:
            raise ValueError(f"static batch holds {self.size} requests, got {n}")
        if n:
            m._prepare_step(handles, 1, False)
        lengths = [h.length for h in handles]
        if n and max(lengths) + 1 > self.max_kv_len:
            raise ValueError("a request outgrew the static batch's max_kv_len")
        m._rows.flush()
        i = self._flip
        self._flip ^= 1
        if self._events[i] is not None:
            self._events[i].synchronize()
        host = self._staging[i]
        pad = self.size - n
        lens = np.asarray(lengths + [0] * pad, dtype=np.int64)
        h = host.numpy()
        h[: 2 * self.size].view(np.int64)[:] = lens
        h[2 * self.size: 3 * self.size] = lens
        h[3 * self.size:] = [handle.slot for handle in handles] + [m.max_requests] * pad
        self.meta.copy_(host, non_blocking=True)
        if m.device.type == "cuda":
            self._events[i] = torch.cuda.Event()
            self._events[i].record()
        torch.index_select(m._rows.dev[:, : self.width], 0, self.meta[3 * self.size:].long(), out=self.table)


class PagedKVCacheManager:
    """Allocate fixed-size, reference-counted pages from shared K/V pools.

    The drop-in for hayate's ``PagedKVCacheManager`` (``hayate/engine/paged_cache.py:74-304``):
    same constructor, methods (``allocate``, ``reserve``, ``truncate``, ``release``,
    ``allocate_for_request``, ``import_cache``, ``snapshot``, ``begin_batch``,
    ``commit_batch``), free-list order and exceptions, plus ``share`` (prefix pages aliased
    with reference counts, copy-on-write on append). Pools are ``[layers, 1, H_kv,
    capacity, head_dim]`` device tensors; ``begin_batch`` returns a ``PagedKVBatch`` whose
    ``write_layer`` / ``attend_layer`` (and ``write_attend_layer``, ``prepare_layer``) run
    this package's kernels.

    Tuning attributes: ``kernel`` pins one attention kernel ("auto" lets the library
    choose), ``split_tokens`` the decode split size (0: the library's), ``prefill_plan``
    turns the prefill schedule on or off and ``prefill_max_splits`` bounds how many items a
    schedule may cut in two. ``check_device_errors()`` raises if a kernel refused input.
    """

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, max_cache_tokens: int,
                 page_size: int, max_requests: int, dtype: torch.dtype,
                 device: torch.device | str):
        if max_cache_tokens < 1:
            raise ValueError("max_cache_tokens must be positive")
        if page_size < 1 or page_size & (page_size - 1):
            raise ValueError("page_size must be a positive power of two")
        if max_requests < 1:
            raise ValueError("max_requests must be positive")
        self.page_size = page_size
        self.num_pages = math.ceil(max_cache_tokens / page_size)
        self.capacity_tokens = self.num_pages * page_size
        self.max_requests = max_requests
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.device = torch.device(device)
        # stacks popped from the end: the lowest slot / page id comes out first
        self._free_slots = list(range(max_requests - 1, -1, -1))
        self._free_pages = list(range(self.num_pages - 1, -1, -1))
        self._page_refs = np.zeros(self.num_pages, dtype=np.int32)
        shape = (num_layers, 1, num_kv_heads, self.capacity_tokens, head_dim)
        self.k_cache = torch.zeros(shape, dtype=dtype, device=self.device)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.error_word = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._workspace: torch.Tensor | None = None
        self._uploader = _MetaUploader(self.device)
        # one row past the request slots: the padding row of fixed-size (graph) batches
        self._rows = _SlotPageTable(max_requests + 1, self.device)
        self._scratch_page: int | None = None
        self.kernel = "auto"     # pin a kernel ("decode", "prefill", "generic") for testing
        self.split_tokens = 0    # 0 lets the library pick the decode split size
        self.prefill_plan = True       # schedule prefill launches (longest first, heaviest split)
        self.prefill_max_splits = 128  # split slots a schedule may use
        self._prefill_ws = None
        self._prefill_ws_zero = 0  # leading bytes of the prefill workspace known to be zero
        self._workspace_zero = 0   # leading bytes of the decode workspace known to be zero
        self._num_sms = None

    # ------------------------------------------------------------------ pages
    def _take_pages(self, count: int) -> list[int]:
        pages = [self._free_pages.pop() for _ in range(count)]
        self._page_refs[pages] = 1
        return pages

    def _drop_pages(self, pages: Sequence[int]) -> None:
        for page in pages:
            self._page_refs[page] -= 1
            if self._page_refs[page] == 0:
                self._free_pages.append(page)

    def page_refcount(self, page: int) -> int:
        return int(self._page_refs[page])

    def allocate(self) -> PagedCacheHandle:
        """Reserve a request slot without allocating KV pages yet."""
        if not self._free_slots:
            raise MemoryError(f"paged cache supports at most {self.max_requests} active requests")
        return PagedCacheHandle(slot=self._free_slots.pop())

    def reserve(self, handle: PagedCacheHandle, required_tokens: int) -> None:
        """Allocate enough pages for ``required_tokens`` logical positions."""
        if handle.released:
            raise RuntimeError("cannot reserve pages for a released cache handle")
        if required_tokens < 0:
            raise ValueError("required_tokens must be non-negative")
        if required_tokens > self.capacity_tokens:
            raise MemoryError(
                f"request needs {required_tokens} cache tokens, but the paged cache "
                f"capacity is {self.capacity_tokens} tokens")
        missing = math.ceil(required_tokens / self.page_size) - len(handle.pages)
        if missing <= 0:
            return
        if len(self._free_pages) < missing:
            raise MemoryError(
                f"paged KV cache is full: need {missing} additional pages, "
                f"but only {len(self._free_pages)} remain")
        new_pages = self._take_pages(missing)
        handle.pages.extend(new_pages)
        self._rows.append(handle.slot, new_pages)

    def share(self, source: PagedCacheHandle, num_tokens: int) -> PagedCacheHandle:
        """New handle whose first ``num_tokens`` alias ``source``'s physical pages.

        No K/V is copied: the pages' reference counts go up. The new request then
        appends into pages of its own (a write into a still-shared page copies it).
        """
        if source.released:
            raise RuntimeError("cannot share pages of a released cache handle")
        if num_tokens < 0 or num_tokens > source.length:
            raise ValueError("shared length must be within the source's cache length")
        handle = self.allocate()
        pages = source.pages[: math.ceil(num_tokens / self.page_size)]
        for page in pages:
            self._page_refs[page] += 1
        handle.pages = list(pages)
        handle.length = num_tokens
        if pages:
            handle.aliased = source.aliased = True
        self._rows.set_row(handle.slot, handle.pages)
        return handle

    def _make_writable(self, handle: PagedCacheHandle, first: int, last: int) -> None:
        """Copy-on-write every page holding logical positions ``first..last`` that is shared."""
        if last < first:
            return
        for logical in range(first // self.page_size, last // self.page_size + 1):
            old = handle.pages[logical]
            if self._page_refs[old] <= 1:
                continue
            if not self._free_pages:
                raise MemoryError("paged KV cache is full: no page left to copy a shared page")
            new = self._take_pages(1)[0]
            size = self.page_size
            for pool in (self.k_cache, self.v_cache):
                pool[:, :, :, new * size:(new + 1) * size].copy_(pool[:, :, :, old * size:(old + 1) * size])
            self._drop_pages([old])
            handle.pages[logical] = new
            self._rows.set_entry(handle.slot, logical, new)

    def allocate_for_request(self, cache=None) -> PagedCacheHandle:
        """Allocate a request handle and optionally import a contiguous prefix."""
        handle = self.allocate()
        try:
            if cache is not None and cache.length:
                self.import_cache(handle, cache)
        except Exception:
            self.release(handle)
            raise
        return handle

    def import_cache(self, handle: PagedCacheHandle, cache) -> None:
        """Copy a contiguous ``[layers, H_kv, tokens, D]`` prefix into the request's pages."""
        if cache.k is None or cache.v is None:
            return
        length = cache.length
        self.reserve(handle, length)
        self._make_writable(handle, 0, length - 1)
        slots = self._physical_positions(handle, length)
        for layer in range(cache.k.shape[0]):
            for pool, src in ((self.k_cache, cache.k), (self.v_cache, cache.v)):
                pool[layer, 0].index_copy_(
                    1, slots, src[layer, :, :length].to(device=pool.device, dtype=pool.dtype))
        handle.length = length

    def truncate(self, handle: PagedCacheHandle, length: int) -> None:
        """Shorten a cache and drop whole pages beyond its new end."""
        if handle.released:
            raise RuntimeError("cannot truncate a released cache handle")
        if length < 0 or length > handle.length:
            raise ValueError("truncate length must be within the current cache length")
        keep = math.ceil(length / self.page_size)
        dropped = handle.pages[keep:]
        handle.pages = handle.pages[:keep]
        self._drop_pages(dropped)
        if dropped:
            self._rows.set_row(handle.slot, handle.pages)
        handle.length = length

    def snapshot(self, handle: PagedCacheHandle, length: int | None = None) -> KVSnapshot:
        """Gather a compact ``[layers, H_kv, length, D]`` copy of a request's cache."""
        if handle.released:
            raise RuntimeError("cannot snapshot a released cache handle")
        n = handle.length if length is None else length
        if n < 0 or n > handle.length:
            raise ValueError("snapshot length must be within the current cache length")
        slots = self._physical_positions(handle, n)
        k = self.k_cache[:, 0].index_select(2, slots).contiguous()
        v = self.v_cache[:, 0].index_select(2, slots).contiguous()
        return KVSnapshot(k, v)

    def release(self, handle: PagedCacheHandle) -> None:
        """Drop a request's pages and return its slot."""
        if handle.released:
            return
        self._drop_pages(handle.pages)
        handle.pages.clear()
        self._rows.set_row(handle.slot, ())
        handle.length = 0
        handle.released = True
        handle.aliased = False
        self._free_slots.append(handle.slot)

    # ------------------------------------------------------------------ steps
    def _prepare_step(self, handles, query_len, packed: bool):
        """Validate a step, reserve its append space and copy shared pages it writes into;
        returns (cache lengths, query lengths, kv lengths) per request."""
        if packed:
            query_lens = [int(n) for n in query_len]
            if len(query_lens) != len(handles):
                raise ValueError("a packed batch needs one query length per request")
        else:
            query_lens = [int(query_len)] * len(handles)
        if min(query_lens) < 1:
            raise ValueError("query_len must be positive")
        if any(handle.released for handle in handles):
            raise RuntimeError("cannot use a released cache handle in an attention batch")
        if len({id(handle) for handle in handles}) != len(handles):
            raise ValueError("an attention batch cannot contain the same cache handle twice")
        if self.page_size < MIN_KV_PAGE_SIZE:
            raise ValueError(f"page_size must be at least {MIN_KV_PAGE_SIZE} tokens")
        size = self.page_size
        lengths = [handle.length for handle in handles]
        kv_lengths = [length + n for length, n in zip(lengths, query_lens)]
        if max(kv_lengths) > self.capacity_tokens:
            raise MemoryError(
                f"request needs more than the paged cache capacity of {self.capacity_tokens} tokens")
        # only requests whose appends cross into a page they do not hold yet need pages
        # (a decode step inside its last page needs none: the common case stays cheap)
        growing = [(h, n) for h, n in zip(handles, kv_lengths) if n > len(h.pages) * size]
        extra = sum(-(-n // size) - len(h.pages) for h, n in growing)
        # plus the pages copy-on-write will take, so that a step that cannot get all of its
        # pages fails here, before any reservation or copy: a held page with r holders that
        # w of this batch's requests append into is copied min(w, r - 1) times (once the
        # others have their copies, the last writer holds it alone)
        writers: dict[int, int] = {}
        for handle, length, n in zip(handles, lengths, query_lens):
            if handle.aliased:
                held_end = min(length + n, len(handle.pages) * size)  # appends into held pages
                for logical in range(length // size, -(-held_end // size)):
                    page = handle.pages[logical]
                    if self._page_refs[page] > 1:
                        writers[page] = writers.get(page, 0) + 1
        extra += sum(min(w, int(self._page_refs[page]) - 1) for page, w in writers.items())
        if extra > len(self._free_pages):
            raise MemoryError(
                f"paged KV cache is full: batch needs {extra} additional pages, "
                f"but only {len(self._free_pages)} remain")
        for handle, target in growing:
            self.reserve(handle, target)
        # copy-on-write where an append lands in a page another request still holds (only
        # requests that took part in share() can hold such pages)
        for handle, length, n in zip(handles, lengths, query_lens):
            if handle.aliased:
                self._make_writable(handle, length, length + n - 1)

        return lengths, query_lens, kv_lengths

    def begin_batch(self, handles: Sequence[PagedCacheHandle],
                    query_len: int | Sequence[int]) -> PagedKVBatch:
        """Reserve append space and upload one step's page table and lengths.

        ``query_len`` is the reference's one chunk length for every request, or a list of
        one length per request: a packed batch, whose new tokens share one token axis
        (prefill chunks of any length and one-token decodes in the same forward pass).
        """
        if not handles:
            raise ValueError("cannot build paged cache metadata for an empty batch")
        packed = not isinstance(query_len, (int, np.integer))
        lengths, query_lens, kv_lengths = self._prepare_step(handles, query_len, packed)

        batch = len(handles)
        width = math.ceil(max(kv_lengths) / self.page_size)
        # page-table rows that changed since the last step, then one small upload:
        # [cache_lens as int64 (2B words) | cache_lens int32 (B) | slots (B)], and for a
        # packed batch [q_start (B) | q_len (B) | decode ids | prefill ids | token rows]
        self._rows.flush()
        slots = [handle.slot for handle in handles]
        if not packed:
            host = np.empty(4 * batch, dtype=np.int32)
            host[: 2 * batch].view(np.int64)[:] = lengths
            host[2 * batch: 3 * batch] = lengths
            host[3 * batch:] = slots
            meta = self._uploader.upload(host)
            table = self._rows.gather(meta[3 * batch:].long(), width)
            return PagedKVBatch(self, table, meta[: 2 * batch].view(torch.int64),
                                meta[2 * batch: 3 * batch], query_len, max(kv_lengths), (meta, table),
                                host_lens=list(lengths))
        q_len = np.asarray(query_lens, dtype=np.int32)
        q_start = np.zeros(batch, dtype=np.int32)
        np.cumsum(q_len[:-1], out=q_start[1:])
        total = int(q_len.sum())
        decode_ids = np.nonzero(q_len == 1)[0].astype(np.int32)
        prefill_ids = np.nonzero(q_len > 1)[0].astype(np.int32)
        token_request = np.repeat(np.arange(batch, dtype=np.int32), q_len)
        n_dec = len(decode_ids)
        host = np.concatenate([np.zeros(2 * batch, dtype=np.int32), np.asarray(lengths, dtype=np.int32),
                               np.asarray(slots, dtype=np.int32), q_start, q_len, decode_ids,
                               prefill_ids, token_request])
        host[: 2 * batch].view(np.int64)[:] = lengths
        meta = self._uploader.upload(host)
        o = 4 * batch
        table = self._rows.gather(meta[3 * batch: o].long(), width)
        layout = PackedLayout(query_lens=query_lens, total_tokens=total,
                              q_start=meta[o: o + batch], q_len=meta[o + batch: o + 2 * batch],
                              decode_ids=meta[o + 2 * batch: o + 2 * batch + n_dec],
                              prefill_ids=meta[o + 2 * batch + n_dec: o + 3 * batch],
                              token_request=meta[o + 3 * batch:])
        return PagedKVBatch(self, table, meta[: 2 * batch].view(torch.int64), meta[2 * batch: 3 * batch],
                            max(query_lens), max(kv_lengths), (meta, table), layout,
                            host_lens=list(lengths))

    def commit_batch(self, handles: Sequence[PagedCacheHandle], query_len: int | Sequence[int]) -> None:
        """Advance logical lengths after every layer wrote the step's K/V."""
        if isinstance(query_len, (int, np.integer)):
            query_lens = [int(query_len)] * len(handles)
        else:
            query_lens = [int(n) for n in query_len]
            if len(query_lens) != len(handles):
                raise ValueError("a packed batch needs one query length per request")
        for handle, n in zip(handles, query_lens):
            if handle.released:
                raise RuntimeError("cannot commit a released cache handle")
            if handle.length + n > len(handle.pages) * self.page_size:
                raise RuntimeError("paged cache append space was not reserved")
            handle.length += n

    # ------------------------------------------------------------------ fixed-size batches
    def _ensure_scratch_page(self) -> None:
        """One page held for good, read and written only by padding rows of fixed-size
        batches (the spare slot row past the request slots points at it)."""
        if self._scratch_page is None:
            if not self._free_pages:
                raise MemoryError("paged KV cache is full: no page left for the padding row")
            self._scratch_page = self._take_pages(1)[0]
            self._rows.set_row(self.max_requests, [self._scratch_page])

    def static_decode_batch(self, size: int, max_kv_len: int, num_q_heads: int) -> StaticDecodeBatch:
        """A fixed-size decode batch for CUDA-graph capture (see ``StaticDecodeBatch``)."""
        return StaticDecodeBatch(self, size, max_kv_len, num_q_heads)

    # ------------------------------------------------------------------ helpers
    def workspace_for(self, batch: int, query_len: int, num_q_heads: int, max_kv_len: int):
        """Grow-only zeroed workspace for the split-KV decode kernel (None if not needed)."""
        need = ops.attention_workspace_bytes(batch, query_len, num_q_heads, self.num_kv_heads,
                                             self.head_dim, max_kv_len, self.k_cache.dtype,
                                             self.split_tokens)
        if need == 0:
            return None
        counters = ops.attention_counter_bytes(batch, self.num_kv_heads)
        if self._workspace is None or self._workspace.numel() < need:
            self._workspace = ops.new_workspace(need, self.device)
        elif counters > self._workspace_zero:
            # this layout's counters reach bytes an earlier, smaller layout used for partials
            self._workspace[self._workspace_zero:counters].zero_()
        # past this layout's counters the bytes may now hold partials; its counters are zero
        # again after every launch
        self._workspace_zero = counters
        return self._workspace

    @property
    def num_sms(self) -> int:
        if getattr(self, "_num_sms", None) is None:
            self._num_sms = (torch.cuda.get_device_properties(self.device).multi_processor_count
                             if self.device.type == "cuda" else 1)
        return self._num_sms

    def prefill_workspace(self, num_splits: int):
        """Grow-only zeroed workspace for split prefill items (None if the plan has none)."""
        need = ops.prefill_workspace_bytes(num_splits)
        if need == 0:
            return None
        counters = ops.prefill_counter_bytes(num_splits)
        if self._prefill_ws is None or self._prefill_ws.numel() < need:
            self._prefill_ws = ops.new_workspace(need, self.device)
        elif counters > self._prefill_ws_zero:
            # more split slots than any layout since the bytes were last known zero: the new
            # counters cover bytes an earlier plan used for partials
            self._prefill_ws[self._prefill_ws_zero:counters].zero_()
        self._prefill_ws_zero = counters
        return self._prefill_ws

    def check_device_errors(self) -> None:
        """Synchronise and raise if a kernel refused a page id or length since the last check."""
        problems = ops.read_device_errors(self.error_word)
        if problems:
            self.error_word.zero_()
            if self._workspace is not None:
                self._workspace.zero_()
            if self._prefill_ws is not None:
                self._prefill_ws.zero_()
            raise RuntimeError("paged attention kernels refused input: " + "; ".join(problems))

    def _physical_positions(self, handle: PagedCacheHandle, length: int) -> torch.Tensor:
        if length == 0:
            return torch.empty(0, dtype=torch.long, device=self.device)
        logical = np.arange(length, dtype=np.int64)
        pages = np.asarray(handle.pages, dtype=np.int64)[logical // self.page_size]
        slots = pages * self.page_size + logical % self.page_size
        return torch.from_numpy(slots).to(self.device)
