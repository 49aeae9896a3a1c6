"""Page copy kernel and the reference's paged-cache behaviours on the B200 classes.

Ports the scenarios of the reference's tests/test_paged_attention.py:47-178 to
the B200 cache (page boundary at 256/257, page reuse after close, mixed
lengths without cross-request reads, snapshot aliasing surviving close, and a
restored prefix continuing exactly like the cache that computed it), with the
oracle standing in for the reference's dense SDPA.
"""

import gc

import pytest
import torch

from helios_b200 import _native
from helios_b200.paged_cache import KVPagePool, PagedBatchCache, PagedKVCache
from oracle.attention import paged_attention
from tests.helpers import attn_config

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _pool(pages=6, layers=2):
    return KVPagePool(attn_config(heads=8, kv_heads=2, layers=layers), pages, device=DEV)


def _tensors(batch, tokens, g):
    return (torch.randn(batch, 8, tokens, 128, generator=g).to(torch.bfloat16).to(DEV),
            (torch.randn(batch, 2, tokens, 128, generator=g) / 3).to(torch.bfloat16).to(DEV),
            torch.randn(batch, 2, tokens, 128, generator=g).to(torch.bfloat16).to(DEV))


def _attend(caches, q, k, v, layer=0):
    batch = PagedBatchCache(caches)
    batch.prepare(q.shape[2])
    out = batch.attend(layer, q, k, v)
    batch.advance(q.shape[2])
    return out, batch


def test_page_copy_copies_every_layer_and_both_pools():
    pool = _pool(pages=8, layers=3)
    g = torch.Generator().manual_seed(0)
    pool.storage.copy_(torch.randn(pool.storage.shape, generator=g).to(torch.bfloat16))
    before = pool.storage.clone()
    pool.copy_pages([1, 6], [4, 0])
    after = pool.storage
    for layer in range(3):
        for kv in range(2):
            assert torch.equal(after[layer, kv, 4], before[layer, kv, 1])
            assert torch.equal(after[layer, kv, 0], before[layer, kv, 6])
            for p in (1, 2, 3, 5, 6, 7):
                assert torch.equal(after[layer, kv, p], before[layer, kv, p])
    assert _native.device_status() == 0
    with pytest.raises(ValueError):
        pool.copy_pages([8], [0])


def test_page_boundary_allocates_the_next_256_token_page():
    pool = _pool()
    g = torch.Generator().manual_seed(1)
    cache = PagedKVCache(pool, 512)
    _attend([cache], *_tensors(1, 256, g))
    assert cache.length == 256 and len(cache.pages) == 1
    first = cache.pages[0].index
    _attend([cache], *_tensors(1, 1, g))
    assert cache.length == 257 and len(cache.pages) == 2
    assert cache.pages[0].index == first and cache.pages[1].index != first


def test_released_page_is_reused_in_a_noncontiguous_batch():
    pool = _pool()
    g = torch.Generator().manual_seed(2)
    first, survivor = PagedKVCache(pool, 512), PagedKVCache(pool, 512)
    _attend([first, survivor], *_tensors(2, 1, g))
    released, survivor_page = first.pages[0].index, survivor.pages[0].index
    first.close()
    replacement = PagedKVCache(pool, 512)
    _attend([replacement], *_tensors(1, 1, g))
    assert replacement.pages[0].index == released != survivor_page
    out, _ = _attend([survivor, replacement], *_tensors(2, 1, g))
    assert out.shape == (2, 8, 1, 128)


def test_mixed_lengths_attend_without_padding_or_cross_request_reads():
    pool = _pool()
    g = torch.Generator().manual_seed(3)
    short, long = PagedKVCache(pool, 512), PagedKVCache(pool, 512)
    for cache, tokens in ((short, 3), (long, 7)):
        _attend([cache], *_tensors(1, tokens, g))
    q, k, v = _tensors(2, 1, g)
    batch = PagedBatchCache([short, long])
    batch.prepare(1)
    assert batch.seqused_k.tolist() == [4, 8]
    assert batch.cu_seq_q.tolist() == [0, 1, 2]
    assert batch.cu_seq_k.tolist() == [0, 4, 12]
    assert batch.block_table.dtype == torch.int32 and batch.cu_seq_k.dtype == torch.int32
    out = batch.attend(0, q, k, v)
    batch.advance(1)
    assert out.shape == (2, 8, 1, 128) and (short.length, long.length) == (4, 8)
    expected = paged_attention(q[:, :, 0].cpu(), pool.keys[0].cpu(), pool.values[0].cpu(),
                               batch.block_table.cpu().tolist(), [0, 1, 2], [4, 8])
    torch.testing.assert_close(out[:, :, 0].cpu().float(), expected.float(), rtol=2e-2, atol=2e-2)


def test_full_page_snapshot_survives_close_and_restores_by_aliasing():
    pool = _pool()
    g = torch.Generator().manual_seed(4)
    cache = PagedKVCache(pool, 512)
    _attend([cache], *_tensors(1, 256, g))
    snapshot = cache.snapshot_block(0, 256)
    page = snapshot.pages[0].index
    cache.close()
    assert pool.free_pages == pool.num_pages - 1
    restored, sibling = PagedKVCache(pool, 512), PagedKVCache(pool, 512)
    restored.restore_blocks([snapshot])
    sibling.restore_blocks([snapshot])
    assert restored.pages[0] is sibling.pages[0] and restored.length == 256
    keys_before = pool.keys[0][page].clone()
    _attend([restored, sibling], *_tensors(2, 1, g))
    assert restored.pages[1].index != sibling.pages[1].index
    assert torch.equal(pool.keys[0][page], keys_before)
    del snapshot
    restored.close()
    sibling.close()
    gc.collect()
    assert pool.free_pages == pool.num_pages


def test_restored_prefix_continuation_matches_the_computing_cache():
    """Aliased pages give the same continuation as the cache that wrote them."""
    pool = _pool(pages=8)
    g = torch.Generator().manual_seed(5)
    writer = PagedKVCache(pool, 300)
    _attend([writer], *_tensors(1, 256, g))
    snap = writer.snapshot_block(0, 256)
    restored = PagedKVCache(pool, 300)
    restored.restore_blocks([snap])
    q, k, v = _tensors(1, 1, g)
    out_w, _ = _attend([writer], q, k, v)
    out_r, _ = _attend([restored], q, k, v)
    torch.testing.assert_close(out_r, out_w, rtol=0, atol=0)
    assert restored.length == 257
