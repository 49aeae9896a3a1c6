"""Tick-packing oracle: the metadata one scheduler tick hands to attention.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Pure Python integers;
the CUDA tick-pack kernel must match these lists bit for bit.

Reference semantics restated here:
  * packed mode -- ``PackedBatchCache.prepare_packed``
    (src/helios/runtime/qwen3/paged_cache.py:418-494)
  * uniform mode -- ``PagedBatchCache.prepare`` (paged_cache.py:221-270)
  * ``_pages_for`` (paged_cache.py:348-349)
"""

from __future__ import annotations

from collections.abc import Sequence


def pages_for(tokens: int, page_size: int) -> int:
    """Pages needed to hold ``tokens`` tokens (paged_cache.py:348-349)."""
    return -(-tokens // page_size)


def pack_tick(
    lengths: Sequence[int],
    counts: Sequence[int],
    page_tables: Sequence[Sequence[int]],
    capacities: Sequence[int],
    *,
    logit_counts: Sequence[int] | None = None,
    page_size: int = 256,
) -> dict:
    """Metadata of a packed mixed tick (paged_cache.py:450-494).

    ``lengths[r]`` is row r's committed KV length before the tick, ``counts[r]``
    its query tokens this tick, ``page_tables[r]`` its page indices *after* the
    pages the tick needs were acquired, ``capacities[r]`` its request capacity.
    """
    rows = len(lengths)
    if logit_counts is None:
        logit_counts = [1] * rows
    offsets = [0]
    for count in counts:
        offsets.append(offsets[-1] + count)
    ends = [length + count for length, count in zip(lengths, counts)]
    width = max(pages_for(cap, page_size) for cap in capacities)
    block_table = [list(table) + [0] * (width - len(table)) for table in page_tables]
    cu_seq_k = [0]
    for end in ends:
        cu_seq_k.append(cu_seq_k[-1] + end)
    positions: list[int] = []
    write_slots: list[int] = []
    for row in range(rows):
        table = page_tables[row]
        for position in range(lengths[row], ends[row]):
            positions.append(position)
            write_slots.append(table[position // page_size] * page_size + position % page_size)
    logit_indices: list[int] = []
    for end, tail in zip(offsets[1:], logit_counts):
        logit_indices.extend(range(end - tail, end))
    return {
        "block_table": block_table,
        "cu_seq_q": offsets,
        "cu_seq_k": cu_seq_k,
        "seqused_k": ends,
        "positions": positions,
        "logit_indices": logit_indices,
        "write_slots": write_slots,
        "max_q": max(counts),
        "max_k": max(ends),
    }


def pack_uniform(
    lengths: Sequence[int],
    tokens: int,
    page_tables: Sequence[Sequence[int]],
    capacities: Sequence[int],
    *,
    page_size: int = 256,
) -> dict:
    """Metadata of a uniform append of ``tokens`` per row (paged_cache.py:241-270).

    ``cu_seq_q`` is ``row * tokens``; no positions or logit rows are produced by
    the reference in this mode (the model derives positions from the lengths).
    """
    out = pack_tick(lengths, [tokens] * len(lengths), page_tables, capacities, page_size=page_size)
    return {
        "block_table": out["block_table"],
        "cu_seq_q": out["cu_seq_q"],
        "cu_seq_k": out["cu_seq_k"],
        "seqused_k": out["seqused_k"],
        "write_slots": out["write_slots"],
        "max_q": tokens,
        "max_k": out["max_k"],
    }
