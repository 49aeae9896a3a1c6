"""Kernel (a) parity: device tick packing vs the reference's metadata, bit for bit.

Every case in ``tests/golden/metadata.json`` was produced by the reference's own
``PagedBatchCache.prepare`` / ``PackedBatchCache.prepare_packed``. The pool is
arranged to hand out the same pages, then the B200 cache's device-built
metadata must equal the reference's lists exactly.
"""

import json
import math

import pytest
import torch

from helios_b200 import _native
from helios_b200.paged_cache import KVPagePool, PackedBatchCache, PagedBatchCache, PagedKVCache
from oracle.metadata import pack_tick
from tests.helpers import attn_config, cache_with_pages, decode_units, queue_pages

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _build(case):
    pages_after = case["page_tables"]
    lengths = case["lengths"]
    before = case.get("pages_before") or [t[: math.ceil(l / 256)] for t, l in zip(pages_after, lengths)]
    num_pages = max([p for t in pages_after for p in t] + [0]) + 8
    pool = KVPagePool(attn_config(heads=4, kv_heads=1), num_pages, device=DEV)
    caches = [cache_with_pages(pool, cap, length, b) for cap, length, b in zip(case["capacities"], lengths, before)]
    queue_pages(pool, [p for t, b in zip(pages_after, before) for p in t[len(b):]])
    return pool, caches


@pytest.mark.parametrize("name", ["ref_mixed_lengths", "ref_prefill_two", "page_boundary", "config1_tick",
                                  "config3_tick", "drafted_rows", "chunked_prefill", "restored_prefix"])
def test_metadata_matches_reference(golden_dir, name):
    case = {c["name"]: c for c in json.loads((golden_dir / "metadata.json").read_text())}[name]
    pool, caches = _build(case)
    if case["mode"] == "uniform":
        batch = PagedBatchCache(caches)
        batch.prepare(case["tokens"])
        keys = ["block_table", "seqused_k", "cu_seq_q", "cu_seq_k", "write_slots"]
    else:
        batch = PackedBatchCache(caches)
        batch.prepare_packed(case["counts"], case["logit_counts"])
        keys = ["block_table", "cu_seq_q", "cu_seq_k", "seqused_k", "positions", "logit_indices", "write_slots"]
    assert [[p.index for p in c.pages] for c in caches] == case["page_tables"]
    for key in keys:
        got = getattr(batch, key)
        expected = case["expected"][key]
        assert got.tolist() == expected, key
        ref_dtype = torch.long if key in ("positions", "logit_indices", "write_slots") else torch.int32
        assert got.dtype == ref_dtype, key
    assert batch.max_q == case["expected"]["max_q"]
    assert batch.max_k == case["expected"]["max_k"]
    assert _native.device_status() == 0


def test_work_items_cover_every_row_once():
    """Decode items tile each decode row's keys by split_keys; prefill items pair query tiles."""
    g = torch.Generator().manual_seed(11)
    pool = KVPagePool(attn_config(heads=32, kv_heads=8), 900, device=DEV)
    lengths = torch.randint(0, 4000, (40,), generator=g).tolist()
    counts = [1] * 30 + [3, 16, 17, 100, 2048, 5, 1, 1, 64, 300]
    caches = []
    for length, count in zip(lengths, counts):
        n = math.ceil(length / 256)
        caches.append(cache_with_pages(pool, length + count + 10, length, [pool._free[-1 - i] for i in range(n)]))
    batch = PackedBatchCache(caches)
    batch.prepare_packed(counts)
    dec = batch.decode_items[: 6 * batch.num_decode_items].view(-1, 6).tolist()
    pre = batch.prefill_items[: 3 * batch.num_prefill_items].view(-1, 3).tolist()
    rec = batch.row_records.tolist()
    group = 4
    seen = {}
    for row, kb, ke, base, n, members in dec:
        assert counts[row] <= 64 // group and members == 0  # no shared pages in this tick
        seen.setdefault(row, []).append((kb, ke, base, n))
    record = 0
    for row, count in enumerate(counts):
        end = lengths[row] + count
        assert rec[row] == record
        if count <= 64 // group:
            items = seen[row]
            units = decode_units(end, batch.split_keys)
            n = len(units)
            assert [(kb, ke) for kb, ke, _, _ in items] == units
            assert all(k == n for _, _, _, k in items)
            assert [b for _, _, b, _ in items] == [record + s * count for s in range(n)]
            record += n * count
        else:
            # Query tiles of 128 // group tokens, adjacent tiles (2i, 2i+1) paired (same key tiles).
            tile = 128 // group
            m = math.ceil(count / tile)
            pairs = [(a, b) for r, a, b in pre if r == row]
            assert pairs == [(2 * i * tile, (2 * i + 1) * tile if 2 * i + 1 < m else -1) for i in range((m + 1) // 2)]
    assert record == batch.partial_records == rec[len(counts)]
    meta = pack_tick(lengths, counts, [[p.index for p in c.pages] for c in caches], [c.capacity for c in caches])
    assert batch.write_slots.tolist() == meta["write_slots"]
    assert batch.token_row.tolist() == [r for r, c in enumerate(counts) for _ in range(c)]
    assert _native.device_status() == 0


def test_second_tick_uploads_only_new_pages_and_restore_resyncs():
    pool = KVPagePool(attn_config(heads=4, kv_heads=1), 16, device=DEV)
    a, b = PagedKVCache(pool, 2000), PagedKVCache(pool, 2000)
    batch = PackedBatchCache([a, b])
    batch.prepare_packed([300, 10])
    batch.advance_packed()
    assert batch._host_descriptor([1, 1], [1, 1])["updates"].size == 0  # no new pages: nothing to upload
    batch.prepare_packed([1, 300])
    assert batch.block_table.tolist() == [[p.index for p in a.pages] + [0] * 6, [p.index for p in b.pages] + [0] * 6]
    batch.advance_packed()
    snap = a.snapshot_block(0, 256)
    c = PagedKVCache(pool, 1000)
    c.restore_blocks([snap])
    batch2 = PackedBatchCache([c])
    batch2.prepare_packed([5])
    assert batch2.block_table.tolist()[0][:2] == [snap.pages[0].index, c.pages[1].index]
    assert batch2.write_slots.tolist() == [c.pages[1].index * 256 + i for i in range(5)]


def test_rows_sharing_restored_pages_form_one_prefix_pass():
    """Single-token decode rows whose page lists start with the same restored pages: the group's
    prefix keys get prefix items once for all its rows (one per split of the shared keys), each
    row keeps decode items for its own keys only, and its records are the prefix splits, then
    its own."""
    pool = KVPagePool(attn_config(heads=32, kv_heads=8), 120, device=DEV)
    prefix = PagedKVCache(pool, 2048)
    prefix.pages.extend(pool.acquire(6))
    prefix.length = 6 * 256
    block = prefix.snapshot_block(0, 6 * 256)
    tails = [40, 300, 700, 5, 256]
    caches = []
    for tail in tails:
        c = PagedKVCache(pool, 4096)
        c.restore_blocks([block])
        c.pages.extend(pool.acquire(math.ceil((6 * 256 + tail) / 256) - 6))
        c.length = 6 * 256 + tail
        caches.append(c)
    other = PagedKVCache(pool, 4096)  # a row with its own pages ends the group
    other.pages.extend(pool.acquire(8))
    other.length = 2000
    batch = PackedBatchCache(caches + [other])
    batch.prepare_packed([1] * 6)
    sk, psk = batch.split_keys, batch.prefix_split_keys
    dec = batch.decode_items[: 6 * batch.num_decode_items].view(-1, 6).tolist()
    pfx = batch.prefix_items[: 5 * batch.num_prefix_items].view(-1, 5).tolist()
    rec = batch.row_records.tolist()
    shared = 6 * 256
    n_prefix = math.ceil(shared / psk)
    assert pfx == [[0, 5, s * psk, min(shared, (s + 1) * psk), s] for s in range(n_prefix)]
    assert all(it[5] == 0 for it in dec)
    for row, tail in enumerate(tails):
        end = shared + tail + 1
        own = [it for it in dec if it[0] == row]
        units = decode_units(end - shared, sk)
        n_own = len(units)
        assert [(kb, ke) for _, kb, ke, _, _, _ in own] == [(shared + a, shared + b) for a, b in units]
        assert [b for _, _, _, b, _, _ in own] == [rec[row] + n_prefix + k for k in range(n_own)]
        assert all(n == n_prefix + n_own for _, _, _, _, n, _ in own)
        assert rec[row + 1] - rec[row] == n_prefix + n_own
    own = [it for it in dec if it[0] == 5]
    assert [(it[1], it[2]) for it in own] == decode_units(2001, sk)  # the unshared row: from key 0
    assert rec[6] == batch.partial_records
    assert _native.device_status() == 0
