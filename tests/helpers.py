"""Shared constructors for the tests: pools, caches holding chosen pages."""

from __future__ import annotations

from collections.abc import Sequence

import torch

from helios_b200.config import Qwen3Config
from helios_b200.paged_cache import KVPage, KVPagePool, PagedKVCache


def attn_config(heads: int = 8, kv_heads: int = 2, head_dim: int = 128, layers: int = 1,
                context: int = 40_960) -> Qwen3Config:
    return Qwen3Config(vocab_size=64, context_length=context, hidden_size=64, n_heads=heads, n_layers=layers,
                       hidden_dim=64, head_dim=head_dim, n_kv_heads=kv_heads, dtype=torch.bfloat16)


def cache_with_pages(pool: KVPagePool, capacity: int, length: int, pages: Sequence[int]) -> PagedKVCache:
    """A request cache of ``length`` tokens that already holds exactly ``pages``."""
    cache = PagedKVCache(pool, capacity)
    for index in pages:
        pool._free.remove(index)
        cache.pages.append(KVPage(pool, index))
    cache.length = length
    return cache


def queue_pages(pool: KVPagePool, pages: Sequence[int]) -> None:
    """Make the pool's next ``acquire`` calls hand out ``pages`` in this order (LIFO list)."""
    for index in pages:
        pool._free.remove(index)
    pool._free.extend(reversed(list(pages)))


def decode_units(keys: int, split: int) -> list[tuple[int, int]]:
    """A decode row's own keys [0, keys) as tick packing cuts them: the nearest whole number of
    ``split`` (at least one) near-equal parts on 64-key boundaries."""
    n = max(1, (keys + split // 2) // split)
    starts = [(keys * k // n) & ~63 for k in range(n)] + [keys]
    return [(starts[k], starts[k + 1]) for k in range(n)]
