"""Paged KV pool and batch caches: the reference's interface over B200 kernels.

Same classes, attributes, methods, argument meaning and exception types as
src/helios/runtime/qwen3/paged_cache.py (``KVPage``, ``PagedKVBlockSnapshot``,
``KVPagePool``, ``PagedKVCache``, ``PagedBatchCache``, ``PackedBatchCache``), so
the decoder, engine and tests written for the reference drive this one. What
changes underneath:

  * the pool is one device allocation ``[layers, {K, V}, pages, page, Hkv, d]``;
    ``keys``/``values`` are the per-layer views the reference exposes
    (paged_cache.py:47-55);
  * each request cache owns a slot in a device-resident *page arena*
    (``int32 [slots, ceil(context / page)]``) mirroring its page list; only pages
    added since the last tick are uploaded;
  * ``prepare``/``prepare_packed`` keep the reference's validation and page
    acquisition on the host (paged_cache.py:221-240, :418-449) but upload one
    small int32 descriptor and let the tick-pack kernel build ``block_table``,
    ``cu_seq_q``, ``cu_seq_k``, ``seqused_k``, ``positions``, ``logit_indices``
    and ``write_slots`` on the device;
  * ``attend`` appends K/V and runs the split-K / tcgen05 paged attention
    kernels instead of ``index_copy_`` + ``varlen_attn`` (paged_cache.py:301-345,
    :501-520). There is no CPU path: a pool that is not on a CUDA device can be
    built and paged (for bookkeeping) but raises on ``attend``.
"""

from __future__ import annotations

import math
import weakref
from collections.abc import Sequence
from dataclasses import dataclass
from itertools import accumulate

import numpy as np
import torch

from helios_b200 import ops
from helios_b200.config import Qwen3Config

DECODE_QUERY_ROWS = 64      # query rows (tokens x group heads) one decode CTA holds
MIN_SHARED_PAGES = 4        # common leading pages from which single-token decode rows share one prefix pass
PREFIX_GROUP_MAX_ROWS = 512  # rows of one shared-prefix group (its prefix items take 2 tiles of rows each)
PREFIX_MIN_SPLIT_KEYS = 512  # shortest split of the shared keys one prefix item covers
PREFIX_SM_SHARE = 4          # the prefix tiles aim at 1/PREFIX_SM_SHARE of the SMs; the decode grid takes the rest
DECODE_SPLIT_CTAS_PER_SM = 8         # decode units per SM the split size aims at (decode-only calls)
DECODE_SPLIT_CTAS_PER_SM_MIXED = 3   # the same when prefill tiles run beside the (persistent) decode grid
PREFILL_TILE_ROWS = 128     # query rows of one tcgen05 prefill tile (a CTA takes a pair of tiles)
NUM_SMS_B200 = 148


class KVPage:
    __slots__ = ("__weakref__", "_finalizer", "index", "pool")

    def __init__(self, pool: "KVPagePool", index: int) -> None:
        self.index = index
        self.pool = pool
        self._finalizer = weakref.finalize(self, pool._release, index)


@dataclass(frozen=True)
class PagedKVBlockSnapshot:
    length: int
    pages: tuple[KVPage, ...]
    memory_bytes: int


def _pages_for(tokens: int, page_size: int) -> int:
    return (tokens + page_size - 1) // page_size


class KVPagePool:
    def __init__(self, config: Qwen3Config, num_pages: int, *, device: torch.device, page_size: int = 256) -> None:
        if num_pages < 1:
            raise ValueError("KV page pool must contain at least one page.")
        if page_size < 1 or page_size % 256:
            raise ValueError("KV page size must be a positive multiple of 256.")
        self.config = config
        self.num_pages = num_pages
        self.page_size = page_size
        self.device = torch.device(device)
        # Zero-filled so no page ever holds NaN bit patterns before its first write.
        self.storage = torch.zeros(
            (config.n_layers, 2, num_pages, page_size, config.n_kv_heads, config.head_dim),
            dtype=config.dtype, device=self.device)
        self.keys = tuple(self.storage[layer, 0] for layer in range(config.n_layers))
        self.values = tuple(self.storage[layer, 1] for layer in range(config.n_layers))
        self._free = list(range(num_pages - 1, -1, -1))
        self.arena_width = _pages_for(config.context_length, page_size)
        self._arena = torch.zeros((0, self.arena_width), dtype=torch.int32, device=self.device)
        self._free_slots: list[int] = []

    @property
    def bytes_per_token(self) -> int:
        return self.config.n_layers * 2 * self.config.n_kv_heads * self.config.head_dim * self.storage.element_size()

    @property
    def bytes_per_page(self) -> int:
        return self.bytes_per_token * self.page_size

    @property
    def free_pages(self) -> int:
        return len(self._free)

    def acquire(self, count: int) -> list[KVPage]:
        if count < 0:
            raise ValueError("Requested page count must not be negative.")
        if count > len(self._free):
            raise RuntimeError(f"KV page pool needs {count} pages but only {len(self._free)} are free.")
        return [KVPage(self, self._free.pop()) for _ in range(count)]

    def _release(self, index: int) -> None:
        self._free.append(index)

    # ---- device page arena (one slot per live request cache)
    @property
    def arena(self) -> torch.Tensor:
        return self._arena

    def _acquire_slot(self) -> int:
        if not self._free_slots:
            old = self._arena.shape[0]
            new = max(64, 2 * old)
            grown = torch.zeros((new, self.arena_width), dtype=torch.int32, device=self.device)
            if old:
                grown[:old].copy_(self._arena)
            self._arena = grown
            self._free_slots = list(range(new - 1, old - 1, -1))
        return self._free_slots.pop()

    def _release_slot(self, slot: int) -> None:
        self._free_slots.append(slot)

    def copy_pages(self, src: Sequence[int], dst: Sequence[int]) -> None:
        """Copy whole pages ``src[i] -> dst[i]`` across every layer's K and V (kernel d)."""
        if len(src) != len(dst):
            raise ValueError("Page copy needs matching source and destination lists.")
        if not src:
            return
        if any(not 0 <= p < self.num_pages for p in (*src, *dst)):
            raise ValueError("Page copy index is outside the pool.")
        pairs = torch.tensor([list(src), list(dst)], dtype=torch.int32).to(self.device)
        flat = self.storage.view(2 * self.config.n_layers, self.num_pages, *self.storage.shape[3:])
        ops.page_copy(flat, pairs[0], pairs[1])


class PagedKVCache:
    batch_size = 1

    def __init__(self, pool: KVPagePool, capacity: int) -> None:
        if not 1 <= capacity <= pool.config.context_length:
            raise ValueError(f"KV-cache capacity must be between 1 and {pool.config.context_length:,} tokens.")
        self.pool = pool
        self.capacity = capacity
        self.pages: list[KVPage] = []
        self.length = 0
        self._pending_tokens: int | None = None
        self._slot = pool._acquire_slot()
        self._synced = 0  # leading page positions whose arena entries are current
        self._slot_finalizer = weakref.finalize(self, pool._release_slot, self._slot)

    @property
    def memory_bytes_per_token(self) -> int:
        return self.pool.bytes_per_token

    @property
    def memory_bytes_per_slot_token(self) -> int:
        return self.pool.bytes_per_token

    def slot_length(self, slot: int) -> int:
        if slot != 0:
            raise ValueError("Single-request paged caches have only slot 0.")
        return self.length

    def snapshot_block_slot(self, slot: int, start: int, end: int) -> PagedKVBlockSnapshot:
        if slot != 0:
            raise ValueError("Single-request paged caches have only slot 0.")
        page_size = self.pool.page_size
        if start < 0 or end <= start or end > self.length or start % page_size or end % page_size:
            raise ValueError("Paged K/V snapshots require complete aligned pages.")
        pages = tuple(self.pages[start // page_size: end // page_size])
        if len(pages) * page_size != end - start:
            raise RuntimeError("Paged K/V snapshot is missing a logical page.")
        return PagedKVBlockSnapshot(length=end - start, pages=pages, memory_bytes=len(pages) * self.pool.bytes_per_page)

    def snapshot_block(self, start: int, end: int) -> PagedKVBlockSnapshot:
        return self.snapshot_block_slot(0, start, end)

    def restore_blocks(self, blocks: Sequence[PagedKVBlockSnapshot]) -> None:
        """Alias the snapshot pages (no bytes move); the arena row is refreshed at the next tick."""
        if self.length or self.pages or self._pending_tokens is not None:
            raise RuntimeError("Paged K/V blocks can only restore into an empty cache.")
        pages: list[KVPage] = []
        for block in blocks:
            if (block.length < 1 or block.length % self.pool.page_size
                    or len(block.pages) * self.pool.page_size != block.length
                    or any(page.pool is not self.pool for page in block.pages)):
                raise ValueError("Paged K/V block does not belong to this aligned pool.")
            pages.extend(block.pages)
        length = len(pages) * self.pool.page_size
        if length > self.capacity:
            raise ValueError("Paged K/V blocks do not fit within this request capacity.")
        self.pages = pages
        self.length = length
        self._synced = 0

    def truncate(self, length: int) -> None:
        if self._pending_tokens is not None or not 0 <= length <= self.length:
            raise ValueError("Cannot truncate beyond committed KV tokens.")
        self.length = length
        del self.pages[_pages_for(length, self.pool.page_size):]
        self._synced = min(self._synced, len(self.pages))

    def close(self) -> None:
        self.pages.clear()
        self.length = 0
        self._pending_tokens = None
        self._synced = 0


class _Staging:
    """Pinned host -> device upload of a tick's int32 descriptor (two pinned buffers
    alternate; an event guards each against reuse before its copy has run)."""

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.host = [torch.empty(0, dtype=torch.int32), torch.empty(0, dtype=torch.int32)]
        self.events: list[torch.cuda.Event | None] = [None, None]
        self.dev = torch.empty(0, dtype=torch.int32, device=device)
        self.turn = 0

    def upload(self, values: np.ndarray) -> torch.Tensor:
        n = int(values.size)
        i = self.turn
        self.turn ^= 1
        if self.events[i] is not None:
            self.events[i].synchronize()
        if self.host[i].numel() < n:
            self.host[i] = torch.empty(max(n, 2 * self.host[i].numel(), 1024), dtype=torch.int32, pin_memory=True)
        if self.dev.numel() < n:
            self.dev = torch.empty(max(n, 2 * self.dev.numel(), 1024), dtype=torch.int32, device=self.device)
        self.host[i].numpy()[:n] = values
        self.dev[:n].copy_(self.host[i][:n], non_blocking=True)
        if self.events[i] is None:
            self.events[i] = torch.cuda.Event()
        self.events[i].record(torch.cuda.current_stream(self.device))
        return self.dev[:n]


def choose_split_keys(decode_keys_x_heads: int, page_size: int, num_sms: int = NUM_SMS_B200,
                      ctas_per_sm: int = DECODE_SPLIT_CTAS_PER_SM) -> int:
    """Keys per decode split: aim for ``ctas_per_sm`` decode units per SM across the decode rows.
    A decode-only call runs one CTA per unit, two per SM, and gains from fine splits that even out
    the rows' lengths (BASELINE config 2's 64 long rows: 170 us at 8 per SM, 174 at 4, 179 at 3).
    Beside prefill tiles the decode grid is persistent on fewer SMs and every unit pays its start
    and merge on those SMs, so fewer, longer units win there (config-3 ticks 18.15 -> 18.03 ms at
    3 per SM; mixed config-3 attention 106.6 -> 102.3 us)."""
    target = ctas_per_sm * num_sms
    split = math.ceil(max(1, decode_keys_x_heads) / target)
    split = max(page_size, math.ceil(split / page_size) * page_size)
    return min(split, 64 * page_size)


def choose_prefix_split_keys(pairs_x_heads: int, max_shared: int, page_size: int, num_sms: int = NUM_SMS_B200) -> int:
    """Keys per split of the shared prefixes. The prefix tiles (one CTA per pair of query tiles,
    split and KV head) run first and the decode grid fills the SMs they leave, so the splits are
    sized for about num_sms / PREFIX_SM_SHARE of those CTAs: few enough that most SMs stream the
    rows' own keys meanwhile, and the tensor-core work of the shared keys ends with them (measured
    at BASELINE config 4, 128 rows on 16 shared pages: 89 / 78 / 74 us for splits of 512 / 1024 /
    2048 keys). At least PREFIX_MIN_SPLIT_KEYS keys, a multiple of the page size."""
    splits = max(1, round(num_sms / PREFIX_SM_SHARE / max(1, pairs_x_heads)))
    split = max(PREFIX_MIN_SPLIT_KEYS, math.ceil(max(1, max_shared) / splits))
    return math.ceil(split / page_size) * page_size


class PagedBatchCache:
    def __init__(self, caches: Sequence[PagedKVCache]) -> None:
        if not caches:
            raise ValueError("Paged batch cache needs at least one request cache.")
        pool = caches[0].pool
        if any(cache.pool is not pool for cache in caches):
            raise ValueError("Paged batch caches must share one KV page pool.")
        if len({id(cache) for cache in caches}) != len(caches):
            raise ValueError("Paged batches require distinct request caches.")
        self._buffers: dict[str, tuple] = {}
        self._metadata_values: dict[str, list] = {}
        self.caches = tuple(caches)
        self.pool = pool
        self.batch_size = len(caches)
        self._staging: _Staging | None = None
        self._i32 = None
        self._i64 = None
        self.workspace: torch.Tensor | None = None
        self.uploaded_bytes = 0
        # Capacity mode (set by the CUDA-graph runner): metadata buffers and attention
        # launches are sized to work capacities with headroom and the kernels read the
        # tick's real work counts from the device, so launch arguments and buffer
        # addresses stay the same from tick to tick.
        self.capacity_mode = False
        self.work_capacity: tuple[int, int, int] | None = None
        self.attention_counts: torch.Tensor | None = None
        self.launch_decode_items = self.launch_prefill_items = self.launch_partial_records = 0
        self.launch_prefix_items = self.num_prefix_items = 0

    @property
    def length(self) -> int:
        if self.batch_size != 1:
            raise RuntimeError("Batched paged caches have independent lengths.")
        return self.caches[0].length

    def slot_ids(self, slots: Sequence[int] | torch.Tensor) -> tuple[int, ...]:
        if isinstance(slots, torch.Tensor):
            if slots.ndim != 1:
                raise ValueError("Paged batch slots must be one-dimensional.")
            rows = tuple(int(value) for value in slots.cpu().tolist())
        else:
            rows = tuple(slots)
        if rows != tuple(range(self.batch_size)):
            raise ValueError("Paged batches require every active cache in order.")
        return rows

    def slot_length(self, slot: int) -> int:
        if not 0 <= slot < self.batch_size:
            raise ValueError("Paged batch slot is outside the active batch.")
        return self.caches[slot].length

    def slot_lengths(self, slots: Sequence[int] | torch.Tensor) -> torch.Tensor:
        rows = self.slot_ids(slots)
        return self.metadata("positions_by_slot", [self.caches[row].length for row in rows], torch.long)

    def prepare(self, tokens: int) -> None:
        if tokens < 1:
            raise ValueError("Paged KV append needs at least one token.")
        page_size = self.pool.page_size
        missing_pages: list[int] = []
        for cache in self.caches:
            if cache._pending_tokens is not None:
                raise RuntimeError("Paged KV cache already has a pending append.")
            end = cache.length + tokens
            if end > cache.capacity:
                raise ValueError("Paged KV append exceeds its request capacity.")
            missing_pages.append(max(0, _pages_for(end, page_size) - len(cache.pages)))
        total_missing = sum(missing_pages)
        if total_missing > self.pool.free_pages:
            raise RuntimeError(
                f"KV page pool needs {total_missing} pages but only {self.pool.free_pages} are free.")
        for cache, missing in zip(self.caches, missing_pages, strict=True):
            if missing:
                cache.pages.extend(self.pool.acquire(missing))
            cache._pending_tokens = tokens
        self._pack([tokens] * self.batch_size, [1] * self.batch_size)
        self.max_q = tokens
        self.max_k = max(cache.length + tokens for cache in self.caches)

    def metadata(self, name: str, values: list, dtype: torch.dtype) -> torch.Tensor:
        """Host/device buffer pair per name, re-uploaded only when values change
        (paged_cache.py:272-288)."""
        shape = (len(values), len(values[0])) if isinstance(values[0], list) else (len(values),)
        cuda = self.pool.device.type == "cuda"
        pair = self._buffers.get(name)
        if pair is None or pair[0].shape != shape:
            host = torch.empty(shape, dtype=dtype, device="cpu", pin_memory=cuda)
            device = torch.empty(shape, dtype=dtype, device=self.pool.device)
            pair = self._buffers[name] = (host, device, torch.cuda.Event() if cuda else None)
        host, device, copied = pair
        if self._metadata_values.get(name) != values:
            if copied is not None:
                copied.synchronize()  # the previous upload from this pinned buffer has run
            host.numpy()[...] = values
            device.copy_(host, non_blocking=cuda)
            if copied is not None:
                copied.record(torch.cuda.current_stream(self.pool.device))
            self._metadata_values[name] = values
        return device

    def advance(self, tokens: int, *, slots: Sequence[int] | torch.Tensor | None = None) -> None:
        if slots is not None:
            self.slot_ids(slots)
        if any(cache._pending_tokens != tokens for cache in self.caches):
            raise RuntimeError("Paged KV advance must match the prepared token count.")
        for cache in self.caches:
            cache.length += tokens
            cache._pending_tokens = None

    # ---------------------------------------------------------------- device metadata
    def _host_descriptor(self, counts: Sequence[int], logit_counts: Sequence[int]) -> dict:
        """Host half of a tick: the int32 row descriptors, the arena entries added since
        the last tick, and the attention work partition. O(rows + new pages)."""
        pool, config = self.pool, self.pool.config
        page_size = pool.page_size
        updates: list[int] = []
        fields: list[int] = []
        for cache, count, lc in zip(self.caches, counts, logit_counts):
            n = len(cache.pages)
            if cache._synced < n:
                slot = cache._slot
                for j in range(cache._synced, n):
                    updates += (slot, j, cache.pages[j].index)
                cache._synced = n
            fields += (cache._slot, cache.length, count, lc, n, 0, 0)
        rows = np.array(fields, dtype=np.int32).reshape(self.batch_size, ops.TICK_ROW_FIELDS)
        group = config.n_heads // config.n_kv_heads
        decode_max = DECODE_QUERY_ROWS // group
        tile_tokens = PREFILL_TILE_ROWS // group
        pair_rows = 2 * tile_tokens
        self._share_prefixes(rows, PREFIX_GROUP_MAX_ROWS)
        ends = rows[:, 1].astype(np.int64) + rows[:, 2]
        cnts = rows[:, 2].astype(np.int64)
        shared = rows[:, 5].astype(np.int64)
        group_rows = rows[:, 6].astype(np.int64)
        heads = group_rows > 0
        is_decode = cnts <= decode_max
        # The decode items read each row's own keys; the prefix items each group's shared keys,
        # once per pair of query tiles.
        mixed = bool((~is_decode).any())  # prefill rows: the decode grid runs beside their tiles
        split = choose_split_keys(int((ends - shared)[is_decode].sum()) * config.n_kv_heads, page_size,
                                  ctas_per_sm=DECODE_SPLIT_CTAS_PER_SM_MIXED if mixed else DECODE_SPLIT_CTAS_PER_SM)
        pairs = (group_rows + pair_rows - 1) // pair_rows
        prefix_split = choose_prefix_split_keys(int(pairs[heads].sum()) * config.n_kv_heads,
                                                int(shared[heads].max(initial=0)), page_size)
        prefix_splits = (shared + prefix_split - 1) // prefix_split
        # Each row's own keys in the nearest whole number of splits, at least one (tick_pack.cuh,
        # tail_split_count): no row ends in a sliver of a split.
        tail_splits = np.maximum(1, (ends - shared + split // 2) // split)
        records = (prefix_splits + tail_splits) * cnts
        return {
            "rows": rows, "updates": np.asarray(updates, dtype=np.int32), "decode_max": decode_max,
            "tile_tokens": tile_tokens, "split_keys": split, "num_decode_items": int(tail_splits[is_decode].sum()),
            "prefix_split_keys": prefix_split, "num_prefix_items": int((pairs * prefix_splits)[heads].sum()),
            "pair_rows": pair_rows, "partial_records": int(records[is_decode].sum()),
            "num_prefill_items": int(((((cnts[~is_decode] + tile_tokens - 1) // tile_tokens) + 1) // 2).sum()),
            "total_tokens": int(cnts.sum()), "num_logits": int(rows[:, 3].sum()),
            "width": _pages_for(max(cache.capacity for cache in self.caches), page_size),
        }

    def _share_prefixes(self, rows: np.ndarray, max_rows: int) -> None:
        """Fill the shared-prefix columns of ``rows``: runs of up to ``max_rows`` consecutive
        single-token decode rows whose page lists start with the same MIN_SHARED_PAGES or more
        pages (restored by aliasing) form a group; every member gets the group's common full
        pages as shared prefix keys and the first member the group size. Their attention reads
        those pages once per pair of tensor-core query tiles (2 x 128 query rows)."""
        page_size = self.pool.page_size
        caches = self.caches
        # Committed pages a row may share: single-token rows only.
        full = np.where(rows[:, 2] == 1, rows[:, 1] // page_size, 0).tolist()
        if max(full, default=0) < MIN_SHARED_PAGES:
            return

        r, count = 0, len(caches)
        while r < count:
            lead = full[r]
            if lead < MIN_SHARED_PAGES:
                r += 1
                continue
            head = caches[r].pages
            common, j = lead, r + 1
            shared = head[:common]  # the group's common pages so far, sliced once per change
            while j < count and j - r < max_rows:
                fj = full[j]
                limit = common if fj >= common else fj
                pages = caches[j].pages
                # Restored pages are the same handle objects, so the slice comparison (element
                # identity first, in C) settles the common case; the index walk finds a shorter
                # common prefix.
                if limit >= MIN_SHARED_PAGES and pages[:limit] == (shared if limit == common else shared[:limit]):
                    lcp = limit
                else:
                    lcp = 0
                    while lcp < limit and pages[lcp].index == head[lcp].index:
                        lcp += 1
                if lcp < MIN_SHARED_PAGES:
                    break
                if lcp != common:
                    common = lcp
                    shared = head[:common]
                j += 1
            if j - r >= 2:
                rows[r:j, 5] = common * page_size
                rows[r, 6] = j - r
                r = j
            else:
                r += 1

    def _pack(self, counts: Sequence[int], logit_counts: Sequence[int]) -> None:
        """Upload the host descriptor and run the tick-pack kernel (kernel a)."""
        pool, config = self.pool, self.pool.config
        if pool.device.type != "cuda":
            raise ValueError("The B200 paged cache needs its pool on a CUDA device.")
        desc = self._host_descriptor(counts, logit_counts)
        self.split_keys = desc["split_keys"]
        self.prefix_split_keys = desc["prefix_split_keys"]
        self.num_decode_items = desc["num_decode_items"]
        self.partial_records = desc["partial_records"]
        self.num_prefill_items = desc["num_prefill_items"]
        self.num_prefix_items = desc["num_prefix_items"]
        if self.capacity_mode:
            cap = self.work_capacity
            if (cap is None or self.num_decode_items > cap[0] or self.num_prefill_items > cap[1]
                    or self.num_prefix_items > cap[2]):
                # Headroom of one more split and one more tile pair per row and twice the prefix
                # items; no prefill or prefix capacity for a tick without them, so its attention
                # runs the decode grid alone (all SMs).
                cap = (self.num_decode_items + self.batch_size,
                       self.num_prefill_items + self.batch_size if self.num_prefill_items else 0,
                       2 * self.num_prefix_items)
                self.work_capacity = cap
            self.launch_decode_items, self.launch_prefill_items, self.launch_prefix_items = cap
            # Each decode item has <= decode_max rows, each prefix item <= pair_rows, one record each.
            self.launch_partial_records = cap[0] * desc["decode_max"] + cap[2] * desc["pair_rows"]
        else:
            self.launch_decode_items, self.launch_prefill_items = self.num_decode_items, self.num_prefill_items
            self.launch_prefix_items = self.num_prefix_items
            self.launch_partial_records = self.partial_records
        rows, updates = desc["rows"], desc["updates"]
        total, width = desc["total_tokens"], desc["width"]
        if self._staging is None:
            self._staging = _Staging(pool.device)
        dev = self._staging.upload(np.concatenate([rows.reshape(-1), updates]))
        self.uploaded_bytes = 4 * (rows.size + updates.size)
        out = self._outputs(self.batch_size, width, total, desc["num_logits"])
        ops.tick_pack(dev[: rows.size], self.batch_size, dev[rows.size:], updates.size // 3, pool.arena,
                      pool.page_size, width, pool.num_pages, desc["decode_max"], desc["split_keys"],
                      desc["tile_tokens"], total, out, prefix_split_keys=desc["prefix_split_keys"])
        need = ops.workspace_bytes(self.launch_partial_records, config.n_heads, config.head_dim)
        if need and (self.workspace is None or self.workspace.numel() < need):
            # Zeroed: its header holds the decode work ticket, which every call leaves at zero.
            self.workspace = torch.zeros(max(need, 2 * (0 if self.workspace is None else self.workspace.numel())),
                                         dtype=torch.uint8, device=pool.device)
        self.block_table = out["block_table"]
        self.cu_seq_q = out["cu_seq_q"]
        self.cu_seq_k = out["cu_seq_k"]
        self.seqused_k = out["seqused_k"]
        self.write_slots = out["write_slots"]
        self.token_positions = out["positions"]
        self.token_row = out["token_row"]
        self.logit_rows = out["logit_indices"]
        self.decode_items = out["decode_items"]
        self.row_records = out["row_records"]
        self.prefill_items = out["prefill_items"]
        self.prefix_items = out["prefix_items"]
        self.attention_counts = out["counts"] if self.capacity_mode else None
        self.total_tokens = total

    def _outputs(self, rows: int, width: int, tokens: int, logits: int) -> dict:
        """Views of two reusable device buffers sized for this tick."""
        n_dec = max(1, self.launch_decode_items)
        n_pre = max(1, self.launch_prefill_items)
        n_pfx = max(1, self.launch_prefix_items)
        sizes32 = [rows * width, rows + 1, rows + 1, rows, max(tokens, 1), ops.DECODE_ITEM_INTS * n_dec, 3 * n_pre, 4,
                   rows + 1, ops.PREFIX_ITEM_INTS * n_pfx]
        sizes64 = [max(tokens, 1), max(tokens, 1), max(logits, 1)]
        dev = self.pool.device
        if self._i32 is None or self._i32.numel() < sum(sizes32):
            self._i32 = torch.empty(2 * sum(sizes32), dtype=torch.int32, device=dev)
        if self._i64 is None or self._i64.numel() < sum(sizes64):
            self._i64 = torch.empty(2 * sum(sizes64), dtype=torch.long, device=dev)
        o32 = list(accumulate(sizes32, initial=0))
        o64 = list(accumulate(sizes64, initial=0))
        v32 = [self._i32[o32[i]:o32[i + 1]] for i in range(len(sizes32))]
        v64 = [self._i64[o64[i]:o64[i + 1]] for i in range(len(sizes64))]
        return {
            "block_table": v32[0].view(rows, width), "cu_seq_q": v32[1], "cu_seq_k": v32[2], "seqused_k": v32[3],
            "token_row": v32[4][:tokens], "decode_items": v32[5], "prefill_items": v32[6], "counts": v32[7],
            "row_records": v32[8], "prefix_items": v32[9],
            "positions": v64[0][:tokens], "write_slots": v64[1][:tokens], "logit_store": v64[2],
            "logit_indices": v64[2][:logits],
        }

    # ---------------------------------------------------------------- attention
    def attend(self, layer: int, queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
        """Reference contract (paged_cache.py:301-333): q ``[B, H, T, d]`` and k/v
        ``[B, Hkv, T, d]`` already normalised and rotated; appends k/v, returns ``[B, H, T, d]``."""
        tokens = _validate_attention_inputs(self, layer, queries, keys, values)
        if any(cache._pending_tokens != tokens for cache in self.caches):
            raise RuntimeError("Call prepare(tokens) before paged attention.")
        out = self._attend_packed(layer, queries.transpose(1, 2).reshape(-1, queries.shape[1], queries.shape[3]),
                                  keys.transpose(1, 2).reshape(-1, keys.shape[1], keys.shape[3]),
                                  values.transpose(1, 2).reshape(-1, values.shape[1], values.shape[3]))
        return out.view(self.batch_size, tokens, queries.shape[1], queries.shape[3]).transpose(1, 2)

    def _attend_packed(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        pool = self.pool
        ops.qk_norm_rope_append(None, k, v, q_scale=None, k_scale=None, eps=0.0, cos=None, sin=None, positions=None,
                                write_slots=self.write_slots, q_out=None, key_pool=pool.keys[layer],
                                value_pool=pool.values[layer])
        q = q.contiguous()
        out = torch.empty_like(q)
        return ops.paged_attention(q, pool.keys[layer], pool.values[layer], self, out)

    def attend_fused(self, layer: int, qkv: torch.Tensor, q_scale: torch.Tensor, k_scale: torch.Tensor, eps: float,
                     cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """The B200 layer path: raw ``qkv [T, (H + 2 Hkv) d]`` from the fused projection
        -> per-head norm + RoPE + KV append (kernel b) -> paged attention (kernel c).
        Returns the attention output ``[T, H, d]``."""
        config, pool = self.pool.config, self.pool
        H, Hkv, d = config.n_heads, config.n_kv_heads, config.head_dim
        tokens = qkv.shape[0]
        if tokens != self.total_tokens:
            raise ValueError("Packed attention expects one flattened token dimension.")
        q = qkv[:, : H * d].view(tokens, H, d)
        k = qkv[:, H * d: (H + Hkv) * d].view(tokens, Hkv, d)
        v = qkv[:, (H + Hkv) * d:].view(tokens, Hkv, d)
        q_rot = torch.empty((tokens, H, d), dtype=qkv.dtype, device=qkv.device)
        ops.qk_norm_rope_append(q, k, v, q_scale=q_scale, k_scale=k_scale, eps=eps, cos=cos, sin=sin,
                                positions=self.token_positions, write_slots=self.write_slots, q_out=q_rot,
                                key_pool=pool.keys[layer], value_pool=pool.values[layer])
        out = torch.empty_like(q_rot)
        return ops.paged_attention(q_rot, pool.keys[layer], pool.values[layer], self, out)


def _validate_attention_inputs(cache: PagedBatchCache, layer: int, queries, keys, values) -> int:
    config = cache.pool.config
    if not 0 <= layer < config.n_layers:
        raise ValueError("Paged attention layer index is outside the model.")
    if (queries.ndim != 4 or keys.ndim != 4 or values.shape != keys.shape
            or queries.shape[0] != cache.batch_size or keys.shape[0] != cache.batch_size
            or queries.shape[1] != config.n_heads or queries.shape[2] != keys.shape[2]
            or queries.shape[-1] != config.head_dim or keys.shape[1] != config.n_kv_heads
            or keys.shape[-1] != config.head_dim):
        raise ValueError("Paged attention tensors do not match the Qwen3 KV shape.")
    return keys.shape[2]


class PackedBatchCache(PagedBatchCache):
    def prepare_packed(self, counts: Sequence[int], logit_counts: Sequence[int] | None = None) -> None:
        if len(counts) != len(self.caches) or any(count < 1 for count in counts):
            raise ValueError("Each packed sequence needs at least one query token.")
        logit_counts = [1] * len(counts) if logit_counts is None else logit_counts
        if len(logit_counts) != len(counts) or any(
                not 1 <= tail <= count for tail, count in zip(logit_counts, counts, strict=True)):
            raise ValueError("Logit rows must be 1 through each sequence length.")
        missing = []
        for cache, count in zip(self.caches, counts, strict=True):
            if cache._pending_tokens is not None or cache.length + count > cache.capacity:
                raise ValueError("Packed append exceeds capacity or an append is pending.")
            missing.append(max(0, _pages_for(cache.length + count, self.pool.page_size) - len(cache.pages)))
        if sum(missing) > self.pool.free_pages:
            raise RuntimeError("Insufficient free pages for packed append.")
        for cache, count, pages in zip(self.caches, counts, missing, strict=True):
            cache.pages.extend(self.pool.acquire(pages))
            cache._pending_tokens = count
        self.counts = tuple(counts)
        self._pack(counts, logit_counts)
        self.positions = self.token_positions.unsqueeze(0)
        self.logit_indices = self.logit_rows
        self.max_q = max(counts)
        self.max_k = max(cache.length + count for cache, count in zip(self.caches, counts, strict=True))

    def advance_packed(self) -> None:
        for cache, count in zip(self.caches, self.counts, strict=True):
            cache.length += count
            cache._pending_tokens = None

    def attend(self, layer: int, queries: torch.Tensor, keys: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
        """Reference contract (paged_cache.py:501-520): ``[1, H, T, d]`` in and out."""
        if queries.shape[0] != 1 or queries.shape[2] != sum(self.counts):
            raise ValueError("Packed attention expects one flattened token dimension.")
        out = self._attend_packed(layer, queries[0].transpose(0, 1), keys[0].transpose(0, 1),
                                  values[0].transpose(0, 1))
        return out.transpose(0, 1).unsqueeze(0)
