"""The attention entry point that allocates nothing, against the regular one.

``hb_paged_attention_static_workspace`` serves callers that cannot allocate device
memory (a host that has handed the whole GPU to its own pool, or a latency-bound
caller that must not pay for cudaMalloc's synchronisation): its split-K partials
live in a fixed array inside the library. Through the C ABI it must give the same
output as ``hb_paged_attention`` with a caller workspace, bit for bit (both run the
same kernels on the same work split), call after call, even though every call
reuses the array the previous call left behind; it must leave the device's memory
use unchanged; and it must refuse work whose partials do not fit the array.

Three launch shapes use the array differently and each is covered: decode rows
beside a prefill row (the persistent decode grid and its work ticket), the same
work with the decode/prefill overlap switched off (one decode CTA per unit), and a
decode-only tick whose long rows split (per-unit decode grid plus the combine).

This file is collected last, so a run that stops at the first failure has
already run every other test.
"""

import ctypes
import math

import pytest
import torch

from helios_b200 import _native, ops
from helios_b200.paged_cache import KVPagePool, PackedBatchCache
from tests.helpers import attn_config, cache_with_pages

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
LIMIT_BYTES = 8 << 20  # HB_STATIC_WORKSPACE_BYTES
DEFAULT_OVERLAP_SMS = 100


def _static_attention(q, key_pool, value_pool, batch, out):
    lib = _native.load()
    return lib.hb_paged_attention_static_workspace(
        q.data_ptr(), key_pool.data_ptr(), value_pool.data_ptr(), key_pool.shape[0], key_pool.shape[1],
        batch.block_table.data_ptr(), batch.block_table.shape[1], batch.cu_seq_q.data_ptr(),
        batch.seqused_k.data_ptr(), batch.batch_size, batch.row_records.data_ptr(),
        batch.decode_items.data_ptr(), batch.num_decode_items,
        batch.prefill_items.data_ptr(), batch.num_prefill_items, batch.prefix_items.data_ptr(), batch.num_prefix_items,
        None, batch.partial_records, batch.split_keys,
        q.shape[0], q.shape[1], key_pool.shape[2], q.shape[2], ctypes.c_float(q.shape[2] ** -0.5),
        out.data_ptr(), torch.cuda.current_stream().cuda_stream)


def _batch(seed, *, prefill=True):
    """Decode rows long enough to split (so the workspace carries partials), with or
    without a prefill row."""
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(2000, 9000, (40,), generator=g).tolist()
    counts = [1] * 36 + [3, 5, 8, 16]
    if prefill:
        lengths, counts = lengths + [0], counts + [200]
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
    return pool, batch, sum(counts)


def _memory():
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0], torch.cuda.memory_stats().get("allocation.all.allocated", 0)


def _check_two_calls(pool, batch, tokens, seed):
    assert batch.partial_records > 0 and batch.num_decode_items > 40  # split rows use the workspace
    need = ops.workspace_bytes(batch.partial_records, 32, 128)
    assert 0 < need <= LIMIT_BYTES
    g = torch.Generator(device=DEV).manual_seed(seed)
    qs = [torch.randn(tokens, 32, 128, device=DEV, generator=g).to(torch.bfloat16) for _ in range(2)]
    wants = [torch.empty_like(q) for q in qs]
    gots = [torch.full_like(q, float("nan")) for q in qs]
    for q, want in zip(qs, wants):
        ops.paged_attention(q, pool.keys[0], pool.values[0], batch, want)
    # One call first, so that everything the library loads lazily is loaded before measuring.
    _native.check(_static_attention(qs[0], pool.keys[0], pool.values[0], batch, gots[0]),
                  "hb_paged_attention_static_workspace")
    before = _memory()
    for q, got in zip(qs, gots):  # the second call reuses what the first left in the array
        got.fill_(float("nan"))
        _native.check(_static_attention(q, pool.keys[0], pool.values[0], batch, got),
                      "hb_paged_attention_static_workspace")
    after = _memory()
    assert after == before, (before, after)
    for got, want in zip(gots, wants):
        assert torch.equal(got, want)
    assert _native.device_status() == 0


def test_static_workspace_matches_caller_workspace_beside_prefill():
    pool, batch, tokens = _batch(0)
    assert batch.num_prefill_items > 0
    _check_two_calls(pool, batch, tokens, 1)


def test_static_workspace_matches_caller_workspace_without_overlap():
    pool, batch, tokens = _batch(3)
    _native.check(_native.load().hb_attention_set_overlap(0), "hb_attention_set_overlap")
    try:
        _check_two_calls(pool, batch, tokens, 4)
    finally:
        _native.check(_native.load().hb_attention_set_overlap(DEFAULT_OVERLAP_SMS), "hb_attention_set_overlap")


def test_static_workspace_matches_caller_workspace_decode_only():
    pool, batch, tokens = _batch(5, prefill=False)
    assert batch.num_prefill_items == 0
    _check_two_calls(pool, batch, tokens, 6)


def test_static_workspace_rejects_partials_beyond_its_size():
    pool, batch, tokens = _batch(2)
    q = torch.zeros(tokens, 32, 128, device=DEV, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    too_many = LIMIT_BYTES // (32 * 129 * 4) + 1  # partial records that would not fit
    lib = _native.load()
    rc = lib.hb_paged_attention_static_workspace(
        q.data_ptr(), pool.keys[0].data_ptr(), pool.values[0].data_ptr(), pool.num_pages, 256,
        batch.block_table.data_ptr(), batch.block_table.shape[1], batch.cu_seq_q.data_ptr(),
        batch.seqused_k.data_ptr(), batch.batch_size, batch.row_records.data_ptr(),
        batch.decode_items.data_ptr(), batch.num_decode_items,
        batch.prefill_items.data_ptr(), batch.num_prefill_items, batch.prefix_items.data_ptr(), batch.num_prefix_items,
        None, too_many, batch.split_keys, tokens, 32, 8, 128,
        ctypes.c_float(0.0883883), out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == _native.HB_ERR_INVALID
    assert "built-in" in _native.last_error()
