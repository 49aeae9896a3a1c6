"""Host-side logic of the B200 paged cache, on CPU (no kernel runs).

Mirrors the reference's error types and messages (paged_cache.py:39-42, :76-83,
:92-96, :116-169, :221-237, :418-446) and checks the tick descriptor the host
uploads: rows, arena updates (only pages added since the last upload) and the
attention work partition.
"""

import gc
import math

import pytest
import torch

from helios_b200.config import Qwen3Config, Sampling
from helios_b200.paged_cache import (
    KVPagePool,
    PackedBatchCache,
    PagedBatchCache,
    PagedKVCache,
    choose_prefix_split_keys,
    choose_split_keys,
    DECODE_SPLIT_CTAS_PER_SM,
    DECODE_SPLIT_CTAS_PER_SM_MIXED,
)

from tests.helpers import decode_units

CPU = torch.device("cpu")


def tiny(**kw) -> Qwen3Config:
    base = dict(vocab_size=64, context_length=4096, hidden_size=16, n_heads=8, n_layers=1, hidden_dim=32,
                head_dim=128, n_kv_heads=2, dtype=torch.bfloat16)
    base.update(kw)
    return Qwen3Config(**base)


def test_pool_validation_and_lifo_pages():
    with pytest.raises(ValueError, match="at least one page"):
        KVPagePool(tiny(), 0, device=CPU)
    with pytest.raises(ValueError, match="multiple of 256"):
        KVPagePool(tiny(), 2, device=CPU, page_size=128)
    pool = KVPagePool(tiny(), 4, device=CPU)
    assert pool.keys[0].shape == (4, 256, 2, 128) and pool.keys[0].dtype == torch.bfloat16
    assert pool.bytes_per_token == 1 * 2 * 2 * 128 * 2
    pages = pool.acquire(2)
    assert [p.index for p in pages] == [0, 1] and pool.free_pages == 2
    with pytest.raises(RuntimeError, match="needs 3 pages but only 2 are free"):
        pool.acquire(3)
    with pytest.raises(ValueError):
        pool.acquire(-1)
    first, second = pages
    del pages
    del second
    del first
    gc.collect()
    assert pool.free_pages == 4
    assert [p.index for p in pool.acquire(1)] == [0]  # LIFO: the last released comes back first


def test_cache_snapshot_restore_truncate_semantics():
    pool = KVPagePool(tiny(), 8, device=CPU)
    with pytest.raises(ValueError, match="capacity must be between"):
        PagedKVCache(pool, 5000)
    cache = PagedKVCache(pool, 1024)
    cache.pages.extend(pool.acquire(3))
    cache.length = 600
    with pytest.raises(ValueError, match="complete aligned pages"):
        cache.snapshot_block(0, 300)
    snap = cache.snapshot_block(0, 512)
    assert snap.length == 512 and len(snap.pages) == 2 and snap.memory_bytes == 2 * pool.bytes_per_page
    other = PagedKVCache(pool, 1024)
    other.restore_blocks([snap])
    assert other.pages[0] is cache.pages[0] and other.length == 512 and other._synced == 0
    with pytest.raises(RuntimeError, match="only restore into an empty cache"):
        other.restore_blocks([snap])
    small = PagedKVCache(pool, 300)
    with pytest.raises(ValueError, match="do not fit"):
        small.restore_blocks([snap])
    cache._synced = 3
    cache.truncate(257)
    assert len(cache.pages) == 2 and cache._synced == 2
    with pytest.raises(ValueError, match="Cannot truncate"):
        cache.truncate(300)
    cache.close()
    assert cache.pages == [] and cache.length == 0


def test_batch_validation_matches_reference_errors():
    pool = KVPagePool(tiny(), 4, device=CPU)
    other_pool = KVPagePool(tiny(), 4, device=CPU)
    a, b = PagedKVCache(pool, 300), PagedKVCache(pool, 300)
    with pytest.raises(ValueError, match="at least one request cache"):
        PagedBatchCache([])
    with pytest.raises(ValueError, match="share one KV page pool"):
        PagedBatchCache([a, PagedKVCache(other_pool, 10)])
    with pytest.raises(ValueError, match="distinct request caches"):
        PagedBatchCache([a, a])
    batch = PackedBatchCache([a, b])
    with pytest.raises(ValueError, match="at least one query token"):
        batch.prepare_packed([1, 0])
    with pytest.raises(ValueError, match="Logit rows"):
        batch.prepare_packed([2, 2], [3, 1])
    with pytest.raises(ValueError, match="exceeds capacity"):
        batch.prepare_packed([1, 400])
    with pytest.raises(RuntimeError, match="Insufficient free pages"):
        PackedBatchCache([PagedKVCache(pool, 2000)]).prepare_packed([1300])
    with pytest.raises(ValueError, match="at least one token"):
        PagedBatchCache([a]).prepare(0)
    with pytest.raises(ValueError, match="exceeds its request capacity"):
        PagedBatchCache([a]).prepare(301)
    with pytest.raises(ValueError, match="every active cache in order"):
        PagedBatchCache([a, b]).slot_ids([1, 0])
    # A CPU pool pages normally but refuses to launch: there is no CPU path.
    with pytest.raises(ValueError, match="CUDA device"):
        PackedBatchCache([a]).prepare_packed([3])
    assert len(a.pages) == 1 and a._pending_tokens == 3


def test_descriptor_uploads_only_new_pages():
    pool = KVPagePool(tiny(), 16, device=CPU)
    a, b = PagedKVCache(pool, 2000), PagedKVCache(pool, 2000)
    a.pages.extend(pool.acquire(2)); a.length = 300
    b.pages.extend(pool.acquire(1)); b.length = 5
    batch = PackedBatchCache([a, b])
    d = batch._host_descriptor([1, 1], [1, 1])
    assert d["rows"].tolist() == [[a._slot, 300, 1, 1, 2, 0, 0], [b._slot, 5, 1, 1, 1, 0, 0]]
    assert d["updates"].reshape(-1, 3).tolist() == [[a._slot, 0, a.pages[0].index], [a._slot, 1, a.pages[1].index],
                                                     [b._slot, 0, b.pages[0].index]]
    assert batch._host_descriptor([1, 1], [1, 1])["updates"].size == 0
    b.pages.extend(pool.acquire(1))
    assert batch._host_descriptor([1, 1], [1, 1])["updates"].tolist() == [b._slot, 1, b.pages[1].index]
    a.truncate(10)
    assert a._synced == 1
    assert a._slot != b._slot


def test_descriptor_partitions_attention_work():
    cfg = tiny(n_heads=32, n_kv_heads=8)
    pool = KVPagePool(cfg, 64, device=CPU)
    caches = []
    for length in (1000, 3000, 0):
        c = PagedKVCache(pool, 4096)
        c.pages.extend(pool.acquire(math.ceil(length / 256)))
        c.length = length
        caches.append(c)
    d = PackedBatchCache(caches)._host_descriptor([1, 16, 2048], [1, 1, 1])
    assert d["decode_max"] == 16 and d["tile_tokens"] == 32
    split = d["split_keys"]
    assert split % 256 == 0 and split >= 256
    n1, n2 = len(decode_units(1001, split)), len(decode_units(3016, split))
    assert d["num_decode_items"] == n1 + n2
    assert d["partial_records"] == n1 * 1 + n2 * 16
    assert d["num_prefill_items"] == 2048 // 32 // 2  # tiles of 32 tokens, paired
    assert d["total_tokens"] == 2065 and d["num_logits"] == 3 and d["width"] == 16


def test_rows_restoring_one_prefix_are_grouped():
    """Consecutive single-token decode rows that restored the same pages form one group: all
    members get the common full pages as shared prefix keys, the first the group size. Rows
    with fewer common pages, several tokens, or their own pages stay alone."""
    cfg = tiny(n_heads=32, n_kv_heads=8)
    pool = KVPagePool(cfg, 128, device=CPU)
    prefix = PagedKVCache(pool, 4096)
    prefix.pages.extend(pool.acquire(8))
    prefix.length = 8 * 256
    full, part = prefix.snapshot_block(0, 8 * 256), prefix.snapshot_block(0, 5 * 256)

    def row(block, tail):
        c = PagedKVCache(pool, 4096)
        c.restore_blocks([block])
        extra = math.ceil((block.length + tail) / 256) - len(c.pages)
        c.pages.extend(pool.acquire(extra))
        c.length = block.length + tail
        return c

    alone = PagedKVCache(pool, 4096)
    alone.pages.extend(pool.acquire(9))
    alone.length = 2100
    caches = [row(full, 10), row(full, 300), row(part, 7), alone, row(full, 3), row(full, 40)]
    counts = [1, 1, 1, 1, 1, 2]
    d = PackedBatchCache(caches)._host_descriptor(counts, [1] * 6)
    rows = d["rows"]
    assert rows[:, 5].tolist() == [5 * 256, 5 * 256, 5 * 256, 0, 0, 0]  # the third row shares 5 pages
    assert rows[:, 6].tolist() == [3, 0, 0, 0, 0, 0]  # row 4 is alone: row 5 has two tokens
    split, prefix_split = d["split_keys"], d["prefix_split_keys"]
    ends = [c.length + n for c, n in zip(caches, counts)]
    shared = 5 * 256
    # The group's shared keys: one prefix item per split (its 3 rows fit one pair of query
    # tiles); each row's own keys: decode items.
    prefix_splits = math.ceil(shared / prefix_split)
    assert prefix_split % 256 == 0 and prefix_split >= 512
    own = [len(decode_units(e - shared, split)) for e in ends[:3]] + [len(decode_units(e, split)) for e in ends[3:]]
    assert d["num_decode_items"] == sum(own)
    assert d["num_prefix_items"] == prefix_splits
    assert d["partial_records"] == 3 * prefix_splits + sum(o * n for o, n in zip(own, counts))


def test_prefix_groups_take_pairs_of_query_tiles():
    """A group of more rows than a pair of tensor-core query tiles holds (2 x 32 tokens at 4
    query heads per KV head) gets one prefix item per pair and split; groups stop at
    PREFIX_GROUP_MAX_ROWS rows."""
    cfg = tiny(n_heads=32, n_kv_heads=8, context_length=8192)
    pool = KVPagePool(cfg, 4096, device=CPU)
    prefix = PagedKVCache(pool, 4096)
    prefix.pages.extend(pool.acquire(16))
    prefix.length = 16 * 256
    block = prefix.snapshot_block(0, prefix.length)
    caches = []
    for tail in range(1, 131):
        c = PagedKVCache(pool, 8192)
        c.restore_blocks([block])
        c.pages.extend(pool.acquire(math.ceil((prefix.length + tail) / 256) - len(c.pages)))
        c.length = prefix.length + tail
        caches.append(c)
    d = PackedBatchCache(caches)._host_descriptor([1] * 130, [1] * 130)
    rows = d["rows"]
    assert rows[:, 6].tolist() == [130] + [0] * 129 and set(rows[:, 5].tolist()) == {4096}
    assert d["pair_rows"] == 64
    splits = math.ceil(4096 / d["prefix_split_keys"])
    assert d["num_prefix_items"] == math.ceil(130 / 64) * splits
    # About a quarter of the SMs run the prefix tiles: 3 pairs x 8 KV heads x 2 splits.
    assert d["prefix_split_keys"] == choose_prefix_split_keys(3 * 8, 4096, 256) == 2048
    # Few rows: more splits of the shared keys; never below PREFIX_MIN_SPLIT_KEYS.
    assert choose_prefix_split_keys(8, 4096, 256) == 1024
    assert choose_prefix_split_keys(1, 1024, 256) == 512


def test_decode_splits_are_longer_beside_prefill():
    """A tick with prefill rows runs its decode grid beside the prefill tiles (persistent, on fewer
    SMs): its split aims at DECODE_SPLIT_CTAS_PER_SM_MIXED units per SM instead of
    DECODE_SPLIT_CTAS_PER_SM, so the same decode rows get splits at least as long."""
    cfg = tiny(n_heads=32, n_kv_heads=8)
    pool = KVPagePool(cfg, 512, device=CPU)
    caches = []
    for length in [1024 + 90 * i for i in range(32)] + [0]:
        c = PagedKVCache(pool, 4096)
        c.pages.extend(pool.acquire(math.ceil(length / 256)))
        c.length = length
        caches.append(c)
    keys_x_heads = sum(c.length + 1 for c in caches[:32]) * 8
    mixed = PackedBatchCache(caches)._host_descriptor([1] * 32 + [2048], [1] * 33)
    alone = PackedBatchCache(caches[:32])._host_descriptor([1] * 32, [1] * 32)
    assert mixed["split_keys"] == choose_split_keys(keys_x_heads, 256, ctas_per_sm=DECODE_SPLIT_CTAS_PER_SM_MIXED)
    assert alone["split_keys"] == choose_split_keys(keys_x_heads, 256, ctas_per_sm=DECODE_SPLIT_CTAS_PER_SM)
    assert mixed["split_keys"] > alone["split_keys"]
    assert mixed["num_decode_items"] < alone["num_decode_items"]


def test_split_policy():
    assert choose_split_keys(0, 256) == 256
    assert choose_split_keys(64 * 4352 * 8, 256) % 256 == 0
    assert choose_split_keys(10 ** 9, 256) == 64 * 256
    # More decode work -> longer splits; never shorter than a page.
    assert choose_split_keys(2 * 10 ** 6, 256) >= choose_split_keys(10 ** 5, 256)


def test_arena_slots_grow_and_recycle():
    pool = KVPagePool(tiny(), 4, device=CPU)
    caches = [PagedKVCache(pool, 10) for _ in range(70)]
    assert pool.arena.shape == (128, math.ceil(4096 / 256))
    slots = {c._slot for c in caches}
    assert len(slots) == 70
    freed = caches[3]._slot
    del caches[3]
    gc.collect()
    assert PagedKVCache(pool, 10)._slot == freed


def test_sampling_bounds_match_reference():
    Sampling(max_new_tokens=1, temperature=0, top_p=1)
    for bad in (dict(max_new_tokens=0), dict(temperature=2.5), dict(top_p=0)):
        with pytest.raises(ValueError):
            Sampling(**bad)


def test_config5_request_distributions():
    """BASELINE config 5's load: lognormal prompts (median 600, sigma 0.8, clipped to
    [16, 8192]), max_new_tokens U[64, 512], Poisson arrivals at the given rate."""
    import numpy as np

    from helios_b200 import load

    reqs = load.make_requests(4000, 151936, seed=5)
    lengths = np.array([len(p) for p, _ in reqs])
    limits = np.array([m for _, m in reqs])
    assert lengths.min() >= 16 and lengths.max() <= 8192
    assert 560 <= np.median(lengths) <= 640
    assert limits.min() >= 64 and limits.max() <= 512 and 270 <= limits.mean() <= 306
    assert all(1 <= t < 151936 for p, _ in reqs[:50] for t in p)  # never the EOS id 0
    arrivals = load.arrival_times(4000, 32.0, seed=5)
    assert np.all(np.diff(arrivals) > 0)
    assert abs(arrivals[-1] / 4000 - 1 / 32.0) < 0.1 / 32.0
    assert load.make_requests(3, 4096, seed=1) == load.make_requests(3, 4096, seed=1)
