"""An immutable K/V snapshot of one request, the value exchanged with hayate's engine.

``PagedKVCacheManager.snapshot`` returns one and ``import_cache`` /
``allocate_for_request`` accept one. hayate only ever reads ``k``, ``v`` and
``length`` from it and takes prefixes with ``slice(end, clone)``: the engine stores
a prompt's snapshot in its prefix cache (``hayate/engine/engine.py:188-198``), the
prefix cache keeps a cloned prefix of it and hands out uncloned prefixes on a hit
(``hayate/engine/prefix_cache.py:57-80``), and the manager copies a hit back into
pages (``hayate/engine/paged_cache.py:142-166``). A snapshot is finished when it is
made, so this type is a read-only view: no in-place growth, no reset. ``extended``
returns a new, longer snapshot for the rare caller that needs one.

Any object with ``k``, ``v`` and ``length`` (hayate's own ``Cache`` included) is
accepted wherever a snapshot is expected.
"""

from __future__ import annotations

import torch


class KVSnapshot:
    """K and V of ``length`` tokens as ``[layers, kv_heads, tokens, head_dim]`` tensors
    (both ``None`` for an empty snapshot). The tensors are shared, not copied, unless a
    method says otherwise."""

    __slots__ = ("_k", "_v")

    def __init__(self, k: torch.Tensor | None = None, v: torch.Tensor | None = None):
        if (k is None) != (v is None):
            raise ValueError("a snapshot holds both K and V or neither")
        if k is not None:
            if k.dim() != 4:
                raise ValueError(f"snapshot tensors are [layers, kv_heads, tokens, head_dim], got {tuple(k.shape)}")
            if k.shape != v.shape:
                raise ValueError(f"snapshot K {tuple(k.shape)} and V {tuple(v.shape)} differ in shape")
        self._k, self._v = k, v

    @classmethod
    def from_tensors(cls, k: torch.Tensor | None, v: torch.Tensor | None) -> "KVSnapshot":
        """Wrap existing tensors (no copy); the token count is their third dimension."""
        return cls(k, v)

    @property
    def k(self) -> torch.Tensor | None:
        return self._k

    @property
    def v(self) -> torch.Tensor | None:
        return self._v

    @property
    def length(self) -> int:
        return 0 if self._k is None else int(self._k.shape[2])

    # a snapshot is exactly as long as it is: no spare room to grow into
    capacity = length

    def slice(self, end: int, clone: bool = False) -> "KVSnapshot":
        """The first ``end`` tokens: a view of these tensors, or compact copies if ``clone``
        (what a prefix cache stores, so later writes to the source cannot reach it)."""
        if not 0 <= end <= self.length:
            raise ValueError(f"prefix of {end} tokens requested from a {self.length}-token snapshot")
        if self._k is None:
            return KVSnapshot()
        k, v = self._k[:, :, :end], self._v[:, :, :end]
        if clone:
            k, v = k.clone(memory_format=torch.contiguous_format), v.clone(memory_format=torch.contiguous_format)
        return KVSnapshot(k, v)

    def extended(self, k: torch.Tensor, v: torch.Tensor) -> "KVSnapshot":
        """A new snapshot with ``k``/``v`` (same layers, heads and head_dim) after these
        tokens. It is one exact-size concatenation: growing token by token this way costs
        a full copy per call, which is why snapshots are made once, from the pages."""
        if self._k is None:
            return KVSnapshot(k, v)
        return KVSnapshot(torch.cat([self._k, k], dim=2), torch.cat([self._v, v], dim=2))

    def __repr__(self) -> str:
        shape = None if self._k is None else tuple(self._k.shape)
        return f"KVSnapshot(length={self.length}, shape={shape})"


# hayate's name for the exchange type (``hayate/model/cache.py``), kept for drop-in use
Cache = KVSnapshot
