"""Kernel (c) parity: paged varlen GQA attention (split-K decode + tcgen05 prefill).

Checked against (1) the reference's own ``PackedBatchCache.attend`` output in
``tests/golden/attention.npz`` and (2) the fp32 oracle on seeded cases covering
decode rows with many splits, drafted rows, partial and multi-tile prefill
rows, chunked-prefill continuation, several GQA group sizes and pools whose
unused slots hold NaN. Tolerance: the reference's own CUDA test bound,
``assert_close(rtol=2e-2, atol=2e-2)`` (tests/test_paged_attention.py:310-312).
"""

import math

import numpy as np
import pytest
import torch

from helios_b200 import _native, ops
from helios_b200.paged_cache import KVPagePool, PackedBatchCache, PagedKVCache
from oracle.attention import paged_attention, write_pool
from tests.golden.inputs import attention_inputs, digest
from tests.helpers import attn_config, cache_with_pages, queue_pages

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def test_matches_reference_packed_attend(golden_dir):
    g = np.load(golden_dir / "attention.npz")
    lengths, counts = g["lengths"].tolist(), g["counts"].tolist()
    key_pool, value_pool, q, k, v = attention_inputs(int(g["num_pages"]), sum(counts))
    assert digest(key_pool, value_pool, q, k, v) == str(g["input_sha256"])
    pool = KVPagePool(attn_config(heads=4, kv_heads=1), int(g["num_pages"]), device=DEV)
    pool.keys[0].copy_(key_pool)
    pool.values[0].copy_(value_pool)
    table = g["block_table"].tolist()
    caches = []
    for row, (length, count) in enumerate(zip(lengths, counts)):
        have = math.ceil(length / 256)
        caches.append(cache_with_pages(pool, length + count + 8, length, table[row][:have]))
    # Hand out the remaining pages exactly as the reference did.
    queue_pages(pool, [p for row, length, count in zip(table, lengths, counts)
                       for p in row[math.ceil(length / 256): math.ceil((length + count) / 256)]])
    batch = PackedBatchCache(caches)
    batch.prepare_packed(counts)
    assert batch.write_slots.tolist() == g["write_slots"].tolist()
    out = batch.attend(0, q.to(DEV), k.to(DEV), v.to(DEV))
    expected = torch.from_numpy(g["out"]).view(torch.bfloat16)
    torch.testing.assert_close(out.cpu().float(), expected.float(), rtol=2e-2, atol=2e-2)
    assert _native.device_status() == 0


def _run(lengths, counts, heads=32, kv_heads=8, seed=0, nan_fill=False):
    g = torch.Generator().manual_seed(seed)
    cfg = attn_config(heads=heads, kv_heads=kv_heads)
    need = sum(math.ceil((l + c) / 256) for l, c in zip(lengths, counts))
    num_pages = need + 4
    pool = KVPagePool(cfg, num_pages, device=DEV)
    fill_k = (torch.randn(pool.keys[0].shape, generator=g) / 3).to(torch.bfloat16)
    fill_v = torch.randn(pool.values[0].shape, generator=g).to(torch.bfloat16)
    order = torch.randperm(num_pages, generator=g).tolist()
    caches, at = [], 0
    for length, count in zip(lengths, counts):
        n = math.ceil(length / 256)
        caches.append(cache_with_pages(pool, length + count + 300, length, order[at: at + n]))
        at += n
    if nan_fill:  # every slot beyond a row's committed context holds NaN
        valid = torch.zeros(num_pages * 256, dtype=torch.bool)
        for c in caches:
            for pos in range(c.length):
                valid[c.pages[pos // 256].index * 256 + pos % 256] = True
        fill_k.view(-1, kv_heads, 128)[~valid] = float("nan")
        fill_v.view(-1, kv_heads, 128)[~valid] = float("nan")
    pool.keys[0].copy_(fill_k)
    pool.values[0].copy_(fill_v)
    batch = PackedBatchCache(caches)
    batch.prepare_packed(counts)
    T = sum(counts)
    q = torch.randn(1, heads, T, 128, generator=g).to(torch.bfloat16)
    k = (torch.randn(1, kv_heads, T, 128, generator=g) / 3).to(torch.bfloat16)
    v = torch.randn(1, kv_heads, T, 128, generator=g).to(torch.bfloat16)
    kp_cpu, vp_cpu = pool.keys[0].cpu(), pool.values[0].cpu()
    out = batch.attend(0, q.to(DEV), k.to(DEV), v.to(DEV))[0].transpose(0, 1).cpu()
    assert _native.device_status() == 0
    slots = batch.write_slots.cpu().tolist()
    write_pool(kp_cpu, slots, k[0].transpose(0, 1))
    write_pool(vp_cpu, slots, v[0].transpose(0, 1))
    expected = paged_attention(q[0].transpose(0, 1).contiguous(), kp_cpu, vp_cpu, batch.block_table.cpu().tolist(),
                               batch.cu_seq_q.cpu().tolist(), batch.seqused_k.cpu().tolist())
    assert torch.isfinite(out.float()).all()
    torch.testing.assert_close(out.float(), expected.float(), rtol=2e-2, atol=2e-2)
    batch.max_abs_err = (out.float() - expected.float()).abs().max().item()
    batch.mean_abs_err = (out.float() - expected.float()).abs().mean().item()
    return batch


def test_decode_rows_split_k():
    g = torch.Generator().manual_seed(1)
    lengths = torch.randint(1, 9000, (48,), generator=g).tolist()
    batch = _run(lengths, [1] * 48)
    assert batch.num_decode_items > 48 and batch.num_prefill_items == 0  # rows were split


def test_decode_rows_short_contexts_and_page_edges():
    _run([0, 1, 63, 64, 65, 255, 256, 257, 511, 512], [1] * 10)


def test_drafted_rows():
    _run([10, 300, 700, 1500, 0, 4000], [2, 3, 5, 8, 16, 16])


def test_prefill_single_row_2048():
    batch = _run([0], [2048])
    assert batch.num_prefill_items == 2048 // 32 // 2  # 64 tiles of 32 tokens, paired
    print(f"prefill 2048 vs fp32 oracle: max abs {batch.max_abs_err:.3e}, mean abs {batch.mean_abs_err:.3e}")
    # Tighter than the reference's bound: one bf16 ulp of the output at most (7.8e-3 measured)
    # and a mean error near bf16 rounding (5.8e-5 measured), so a worse exponential or a dropped
    # key shows up here before it reaches the 2e-2 parity bound.
    assert batch.max_abs_err <= 1.6e-2 and batch.mean_abs_err <= 2e-4


def test_prefill_partial_tiles_and_continuation():
    _run([0, 0, 1000, 256, 77], [17, 33, 300, 150, 100])


def test_mixed_tick():
    g = torch.Generator().manual_seed(3)
    lengths = torch.randint(1024, 4097, (32,), generator=g).tolist() + [0]
    _run(lengths, [1] * 32 + [512])


def test_mixed_tick_is_complete_for_work_queued_after_it():
    """A tick with both halves of the work list, called on a non-default stream: work the
    caller queues right behind it on that stream sees every output row written, call after call."""
    g = torch.Generator().manual_seed(9)
    lengths = torch.randint(1024, 4097, (32,), generator=g).tolist() + [0]
    counts = [1] * 32 + [2048]
    pages = sum(math.ceil((l + c) / 256) for l, c in zip(lengths, counts)) + 4
    pool = KVPagePool(attn_config(heads=32, kv_heads=8), pages, device=DEV)
    pool.storage.normal_(0.0, 0.3)
    order = torch.randperm(pages, generator=g).tolist()
    caches, at = [], 0
    for length, count in zip(lengths, counts):
        n = math.ceil(length / 256)
        caches.append(cache_with_pages(pool, length + count + 8, length, order[at: at + n]))
        at += n
    batch = PackedBatchCache(caches)
    batch.prepare_packed(counts)
    assert batch.num_decode_items > 0 and batch.num_prefill_items > 0
    q = torch.randn(sum(counts), 32, 128, device=DEV).to(torch.bfloat16)
    want = torch.empty_like(q)
    ops.paged_attention(q, pool.keys[0], pool.values[0], batch, want)
    torch.cuda.synchronize()
    assert torch.isfinite(want.float()).all()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    snaps = []
    with torch.cuda.stream(stream):
        out = torch.empty_like(q)
        for _ in range(3):
            out.fill_(float("nan"))
            ops.paged_attention(q, pool.keys[0], pool.values[0], batch, out)
            snaps.append(out.clone())  # queued right behind the attention call
    torch.cuda.synchronize()
    for snap in snaps:
        assert torch.equal(snap, want)
    assert _native.device_status() == 0


@pytest.mark.parametrize("heads,kv_heads", [(8, 8), (16, 8), (64, 8)])
def test_other_group_sizes(heads, kv_heads):
    _run([100, 1000, 0, 300], [1, 4, 200, 40], heads=heads, kv_heads=kv_heads)


def test_stale_nan_slots_never_reach_the_output():
    _run([5, 300, 0, 600], [1, 2, 70, 1], nan_fill=True)


@pytest.mark.parametrize("budget", [1, 7, 100])
def test_persistent_decode_beside_prefill_matches_per_unit_decode(budget):
    """With prefill work in the call the decode rows run on the persistent grid, which keeps
    `budget` SMs (hb_attention_set_overlap). Decode rows of 1, 4, 8 and 16 tokens (16, 32 and
    64 query rows per KV head: every key-split mode), single- and multi-split, give the same
    bits as the one-CTA-per-unit grid (budget 0), call after call (the work ticket is reset
    between calls), and the oracle's values."""
    g = torch.Generator().manual_seed(5)
    lengths = torch.randint(1, 6000, (24,), generator=g).tolist() + [0, 700]
    counts = [1] * 12 + [4] * 4 + [8] * 4 + [16] * 4 + [300, 200]
    lib = _native.load()
    try:
        _native.check(lib.hb_attention_set_overlap(0), "hb_attention_set_overlap")
        base = _run(lengths, counts, seed=5)
        want = base.attend(0, *_qkv(base, 5))
        _native.check(lib.hb_attention_set_overlap(budget), "hb_attention_set_overlap")
        batch = _run(lengths, counts, seed=5)
        for _ in range(2):
            got = batch.attend(0, *_qkv(batch, 5))
            assert torch.equal(got, want)
        assert _native.device_status() == 0
    finally:
        _native.check(lib.hb_attention_set_overlap(100), "hb_attention_set_overlap")
    assert batch.num_prefill_items > 0 and batch.num_decode_items > 24


def _qkv(batch, seed):
    """Fresh q/k/v for another attend on the same prepared batch (same values for a seed)."""
    g = torch.Generator().manual_seed(seed + 1000)
    T = batch.total_tokens
    q = torch.randn(1, 32, T, 128, generator=g).to(torch.bfloat16).to(DEV)
    k = (torch.randn(1, 8, T, 128, generator=g) / 3).to(torch.bfloat16).to(DEV)
    v = torch.randn(1, 8, T, 128, generator=g).to(torch.bfloat16).to(DEV)
    return q, k, v


def _shared_prefix_batch(tails, prefix_pages, extra_counts=(), seed=7, heads=32, kv_heads=8):
    """Rows that restored one prefix snapshot (page aliasing) plus their own tails, one query
    token each, then rows with `extra_counts` tokens and no shared pages."""
    g = torch.Generator().manual_seed(seed)
    cfg = attn_config(heads=heads, kv_heads=kv_heads)
    need = prefix_pages + sum(math.ceil((prefix_pages * 256 + t + 1) / 256) - prefix_pages for t in tails)
    need += sum(math.ceil((c + 300) / 256) for c in extra_counts) + 4
    pool = KVPagePool(cfg, need, device=DEV)
    pool.keys[0].copy_((torch.randn(pool.keys[0].shape, generator=g) / 3).to(torch.bfloat16))
    pool.values[0].copy_(torch.randn(pool.values[0].shape, generator=g).to(torch.bfloat16))
    prefix = PagedKVCache(pool, prefix_pages * 256)
    prefix.pages.extend(pool.acquire(prefix_pages))
    prefix.length = prefix_pages * 256
    block = prefix.snapshot_block(0, prefix.length)
    caches = []
    for tail in tails:
        c = PagedKVCache(pool, prefix.length + tail + 16)
        c.restore_blocks([block])
        c.pages.extend(pool.acquire(math.ceil((prefix.length + tail) / 256) - prefix_pages))
        c.length = prefix.length + tail
        caches.append(c)
    for count in extra_counts:
        c = PagedKVCache(pool, count + 600)
        c.pages.extend(pool.acquire(1))
        c.length = 256
        caches.append(c)
    batch = PackedBatchCache(caches)
    batch.prepare_packed([1] * len(tails) + list(extra_counts))
    return pool, batch, prefix


@pytest.mark.parametrize("tails,prefix_pages,extra,heads", [
    ([10, 300, 700, 5, 256, 1000], 16, (), 32),              # decode grid per unit, then the prefix tiles
    ([40] * 20, 6, (), 32),                                  # 20 rows: one pair of query tiles
    ([3, 500, 77, 1200, 64], 9, (700,), 32),                # beside a prefill row: the persistent grid
    ([(7 * i) % 1000 + 1 for i in range(130)], 16, (), 32),  # 130 rows: 3 pairs, several prefix splits
    ([(11 * i) % 500 + 1 for i in range(70)], 8, (), 8),     # 1 query head per KV head: 128-token tiles
    ([(13 * i) % 300 + 1 for i in range(40)], 5, (300,), 64),  # 8 query heads per KV head: 16-token tiles
])
def test_rows_sharing_a_prefix_match_the_oracle(tails, prefix_pages, extra, heads):
    pool, batch, prefix = _shared_prefix_batch(tails, prefix_pages, extra, heads=heads)
    assert batch.num_prefix_items > 0  # the prefix is read once per pair of query tiles
    g = torch.Generator().manual_seed(99)
    T = batch.total_tokens
    q = torch.randn(1, heads, T, 128, generator=g).to(torch.bfloat16)
    k = (torch.randn(1, 8, T, 128, generator=g) / 3).to(torch.bfloat16)
    v = torch.randn(1, 8, T, 128, generator=g).to(torch.bfloat16)
    kp_cpu, vp_cpu = pool.keys[0].cpu(), pool.values[0].cpu()
    out = batch.attend(0, q.to(DEV), k.to(DEV), v.to(DEV))[0].transpose(0, 1).cpu()
    assert _native.device_status() == 0
    slots = batch.write_slots.cpu().tolist()
    write_pool(kp_cpu, slots, k[0].transpose(0, 1))
    write_pool(vp_cpu, slots, v[0].transpose(0, 1))
    expected = paged_attention(q[0].transpose(0, 1).contiguous(), kp_cpu, vp_cpu, batch.block_table.cpu().tolist(),
                               batch.cu_seq_q.cpu().tolist(), batch.seqused_k.cpu().tolist())
    assert torch.isfinite(out.float()).all()
    torch.testing.assert_close(out.float(), expected.float(), rtol=2e-2, atol=2e-2)


def test_config2_exact_inputs_match_oracle():
    """BASELINE config 2 exactly as the bench times it (helios_b200.workloads.config2_batch:
    seed 1, 64 rows x 1 query, contexts U[512, 8192], pages from a permutation of a
    4096-page pool) against the fp32 oracle, row by row."""
    from helios_b200.workloads import config2_batch

    pool, batch, q, contexts = config2_batch(DEV)
    out = torch.empty_like(q)
    with torch.inference_mode():
        ops.paged_attention(q, pool.keys[0], pool.values[0], batch, out)
    torch.cuda.synchronize()
    assert batch.seqused_k.tolist() == contexts
    want = paged_attention(q.cpu(), pool.keys[0].cpu(), pool.values[0].cpu(), batch.block_table.cpu().tolist(),
                           batch.cu_seq_q.cpu().tolist(), contexts)
    got = out.cpu().float()
    err = (got - want.float()).abs()
    print(f"config 2 decode attention vs oracle: max abs {err.max().item():.3e}, "
          f"max |out| {want.float().abs().max().item():.3e}")
    torch.testing.assert_close(got, want.float(), rtol=1e-2, atol=1e-4)
    assert _native.device_status() == 0
