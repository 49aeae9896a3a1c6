"""Causal paged GQA attention oracle over a pool of fixed-size KV pages.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates the reference's CPU branch of ``PackedBatchCache.attend``
(src/helios/runtime/qwen3/paged_cache.py:521-546) and ``_gather_cpu``
(:405-414): for every row, gather its pages up to ``seqused_k``, repeat each KV
head over its group of query heads (``repeat_interleave``, :527-531), mask
``key_pos <= row_length + i`` (bottom-right causal, :532-535) and run softmax
attention with scale ``1/sqrt(head_dim)`` (SDPA default). Scores, softmax and the
weighted sum are computed in fp32 and rounded once to the query dtype.

Also restates the write step ``PagedBatchCache._write`` (:335-345): packed
``[T, Hkv, d]`` rows land at ``write_slots`` of the flattened pool.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch


def write_pool(pool: torch.Tensor, write_slots: Sequence[int], rows: torch.Tensor) -> None:
    """``pool.view(-1, Hkv, d).index_copy_(0, slots, rows)`` (paged_cache.py:340-345)."""
    flat = pool.view(-1, pool.shape[-2], pool.shape[-1])
    flat.index_copy_(0, torch.as_tensor(list(write_slots), dtype=torch.long), rows.to(pool.dtype))


def gather_row(pool: torch.Tensor, pages: Sequence[int], length: int) -> torch.Tensor:
    """Row's first ``length`` tokens as ``[Hkv, length, d]`` (paged_cache.py:405-414)."""
    index = torch.as_tensor(list(pages), dtype=torch.long)
    return pool.index_select(0, index).reshape(-1, pool.shape[-2], pool.shape[-1])[:length].permute(1, 0, 2)


def paged_attention(
    queries: torch.Tensor,
    key_pool: torch.Tensor,
    value_pool: torch.Tensor,
    block_table: Sequence[Sequence[int]],
    cu_seq_q: Sequence[int],
    seqused_k: Sequence[int],
    *,
    scale: float | None = None,
) -> torch.Tensor:
    """Packed queries ``[T, H, d]`` -> output ``[T, H, d]`` in the query dtype.

    Row r owns query tokens ``cu_seq_q[r]:cu_seq_q[r+1]`` and keys
    ``0:seqused_k[r]``; query i of row r sits at key position
    ``seqused_k[r] - count_r + i``.
    """
    tokens, heads, dim = queries.shape
    kv_heads = key_pool.shape[-2]
    group = heads // kv_heads
    if group * kv_heads != heads:
        raise ValueError("Query heads must be a multiple of KV heads for GQA.")
    scale = dim ** -0.5 if scale is None else scale
    page_size = key_pool.shape[1]
    out = torch.empty(tokens, heads, dim, dtype=queries.dtype)
    for row in range(len(seqused_k)):
        start, stop = cu_seq_q[row], cu_seq_q[row + 1]
        count = stop - start
        if count == 0:
            continue
        end = seqused_k[row]
        pages = list(block_table[row])[: -(-end // page_size)]
        keys = gather_row(key_pool, pages, end).float().repeat_interleave(group, dim=0)
        values = gather_row(value_pool, pages, end).float().repeat_interleave(group, dim=0)
        q = queries[start:stop].float().permute(1, 0, 2)  # [H, count, d]
        scores = torch.matmul(q, keys.transpose(1, 2)) * scale
        key_pos = torch.arange(end)
        query_pos = end - count + torch.arange(count)
        mask = key_pos[None, :] <= query_pos[:, None]
        scores = scores.masked_fill(~mask[None], float("-inf"))
        probs = torch.softmax(scores, dim=-1)
        out[start:stop] = torch.matmul(probs, values).permute(1, 0, 2).to(queries.dtype)
    return out


def attention_partials(
    queries: torch.Tensor,
    key_pool: torch.Tensor,
    value_pool: torch.Tensor,
    pages: Sequence[int],
    key_start: int,
    key_stop: int,
    row_end: int,
    *,
    scale: float,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Unnormalised split of one row over keys ``[key_start, key_stop)``.

    Returns ``(lse[H, count], out[H, count, d])`` with ``out`` normalised within
    the split; combining splits by ``exp(lse)`` weights gives the full softmax.
    Used to check the split-K combine step on its own.
    """
    count = queries.shape[0]
    heads, kv_heads = queries.shape[1], key_pool.shape[-2]
    group = heads // kv_heads
    keys = gather_row(key_pool, pages, row_end)[:, key_start:key_stop].float().repeat_interleave(group, 0)
    values = gather_row(value_pool, pages, row_end)[:, key_start:key_stop].float().repeat_interleave(group, 0)
    q = queries.float().permute(1, 0, 2)
    scores = torch.matmul(q, keys.transpose(1, 2)) * scale
    key_pos = torch.arange(key_start, key_stop)
    query_pos = row_end - count + torch.arange(count)
    scores = scores.masked_fill(~(key_pos[None, :] <= query_pos[:, None])[None], float("-inf"))
    lse = torch.logsumexp(scores, dim=-1)
    out = torch.matmul(torch.softmax(scores, dim=-1), values)
    return lse, out
