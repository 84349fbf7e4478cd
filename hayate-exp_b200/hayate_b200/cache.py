"""Contiguous per-request K/V snapshot, the exchange type of ``import_cache``/``snapshot``.

Same interface as hayate's ``Cache`` (``hayate/model/cache.py:6-83``): tensors of
shape ``[layers, KV heads, tokens, head_dim]``, ``length``/``capacity``,
``from_tensors``, ``append``, ``slice`` and ``reset``. Any object exposing
``k``, ``v`` and ``length`` (the reference's own ``Cache`` included) is accepted
where one is expected.
"""

from __future__ import annotations

import torch


class Cache:
    __slots__ = ("k", "v", "_length")

    def __init__(self):
        self.k: torch.Tensor | None = None
        self.v: torch.Tensor | None = None
        self._length = 0

    @classmethod
    def from_tensors(cls, k: torch.Tensor | None, v: torch.Tensor | None) -> "Cache":
        cache = cls()
        cache.k, cache.v = k, v
        cache._length = 0 if k is None else k.shape[2]
        return cache

    @property
    def length(self) -> int:
        return self._length

    @property
    def capacity(self) -> int:
        return 0 if self.k is None else self.k.shape[2]

    def append(self, k: torch.Tensor, v: torch.Tensor, capacity: int | None = None) -> None:
        if k.shape != v.shape:
            raise ValueError("key and value cache tensors must have matching shapes")
        added = k.shape[2]
        if added == 0:
            return
        need = self._length + added
        if self.k is None or self.v is None or self.capacity < need:
            grown = max(need, capacity or 0, max(1, 2 * self.capacity))
            shape = (k.shape[0], k.shape[1], grown, k.shape[3])
            new_k = torch.empty(shape, dtype=k.dtype, device=k.device)
            new_v = torch.empty(shape, dtype=v.dtype, device=v.device)
            if self.k is not None and self.v is not None and self._length:
                new_k[:, :, : self._length].copy_(self.k[:, :, : self._length])
                new_v[:, :, : self._length].copy_(self.v[:, :, : self._length])
            self.k, self.v = new_k, new_v
        self.k[:, :, self._length : need].copy_(k)
        self.v[:, :, self._length : need].copy_(v)
        self._length = need

    def slice(self, end: int, clone: bool = False) -> "Cache":
        if end < 0:
            raise ValueError("cache slice end must be non-negative")
        if self.k is None or self.v is None:
            return Cache()
        if end > self.length:
            raise ValueError(f"cache slice end {end} exceeds cache length {self.length}")
        k, v = self.k[:, :, :end], self.v[:, :, :end]
        if clone:
            k, v = k.contiguous().clone(), v.contiguous().clone()
        return Cache.from_tensors(k, v)

    def reset(self) -> None:
        self.k = self.v = None
        self._length = 0
