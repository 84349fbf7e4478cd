"""Seeded synthetic inputs with hayate's Qwen3-4B attention statistics.

Q, K and V are N(0, 1); Q and K then get the per-head RMSNorm (weight 1,
eps 1e-6) of ``hayate/model/attention.py:34-35,62-63`` and the half-split RoPE
of ``hayate/model/rope.py:4-47`` (theta 1e6, fp32 tables, result cast back to
the input dtype) at each token's true logical position. V is left as drawn.
Page tables come from a seeded shuffle of the manager's free-page stack.
"""

from __future__ import annotations

import random

import torch

from .paged_cache import PagedCacheHandle, PagedKVCacheManager

ROPE_THETA = 1_000_000.0
QWEN3_4B = dict(num_q_heads=32, num_kv_heads=8, head_dim=128)


def rope_angles(positions: torch.Tensor, head_dim: int, theta: float = ROPE_THETA) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin ``[len(positions), head_dim]`` with the frequency list repeated over both halves."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32,
                                             device=positions.device) / head_dim))
    angles = positions.to(torch.float32)[:, None] * inv_freq[None, :]
    angles = torch.cat([angles, angles], dim=1)
    return torch.cos(angles), torch.sin(angles)


def apply_rope(x: torch.Tensor, positions: torch.Tensor, theta: float = ROPE_THETA) -> torch.Tensor:
    """Rotate ``x`` ``[..., tokens, head_dim]`` by its tokens' positions (``[tokens]``)."""
    head_dim = x.shape[-1]
    cos, sin = rope_angles(positions, head_dim, theta)
    half = head_dim // 2
    rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return (x * cos + rotated * sin).to(x.dtype)


def qk_norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


def qk_tokens(shape, positions: torch.Tensor, dtype, device, gen: torch.Generator) -> torch.Tensor:
    """N(0,1) → RMSNorm → RoPE, shape ``[..., tokens, head_dim]``."""
    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype)
    return apply_rope(qk_norm(x), positions)


def v_tokens(shape, dtype, device, gen: torch.Generator) -> torch.Tensor:
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype)


def shuffle_free_pages(manager: PagedKVCacheManager, seed: int) -> None:
    random.Random(seed).shuffle(manager._free_pages)


def fill_history(manager: PagedKVCacheManager, handle: PagedCacheHandle, length: int,
                 gen: torch.Generator, layers=None, chunk: int = 8192, start: int = 0) -> None:
    """Give ``handle`` tokens ``start .. length - 1`` of synthetic K/V (written into its pages).

    With ``start > 0`` the first ``start`` tokens are kept (e.g. a shared prefix).
    """
    manager.reserve(handle, length)
    device, dtype = manager.k_cache.device, manager.k_cache.dtype
    H, D, P = manager.num_kv_heads, manager.head_dim, manager.page_size
    layers = range(manager.num_layers) if layers is None else layers
    pages = torch.tensor(handle.pages, dtype=torch.int64, device=device)
    for first in range(start, length, chunk):
        stop = min(length, first + chunk)
        pos = torch.arange(first, stop, device=device)
        slots = pages[pos // P] * P + pos % P
        for layer in layers:
            k = qk_tokens((H, stop - first, D), pos, dtype, device, gen)
            v = v_tokens((H, stop - first, D), dtype, device, gen)
            manager.k_cache[layer, 0].index_copy_(1, slots, k)
            manager.v_cache[layer, 0].index_copy_(1, slots, v)
    handle.length = length


def step_inputs(manager: PagedKVCacheManager, handles, query_len: int, num_q_heads: int,
                gen: torch.Generator, strided: bool = True, lengths=None):
    """q ``[B, H_q, T, D]`` and new k/v ``[B, H_kv, T, D]`` for one step at true positions.

    With ``strided`` the tensors are ``[B, T, H, D]`` memory viewed as
    ``[B, H, T, D]``, the layout hayate's attention module hands over. ``lengths``
    overrides the handles' current lengths (inputs for a later step).
    """
    device, dtype = manager.k_cache.device, manager.k_cache.dtype
    H, D = manager.num_kv_heads, manager.head_dim
    B = len(handles)
    lens = torch.tensor([h.length for h in handles] if lengths is None else list(lengths), device=device)
    pos = lens[:, None] + torch.arange(query_len, device=device)[None, :]  # [B, T]

    def make(heads, is_qk):
        x = torch.randn((B, query_len, heads, D), generator=gen, device=device,
                        dtype=torch.float32).to(dtype)
        if is_qk:
            cos, sin = rope_angles(pos.reshape(-1), D)
            cos = cos.view(B, query_len, 1, D)
            sin = sin.view(B, query_len, 1, D)
            x = qk_norm(x)
            half = D // 2
            rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
            x = (x * cos + rotated * sin).to(dtype)
        x = x.transpose(1, 2)
        return x if strided else x.contiguous()

    return make(num_q_heads, True), make(H, True), make(H, False)
