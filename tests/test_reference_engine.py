"""The reference's Engine over this package's decoder, page pool and caches (host side).

``helios_b200.reference_engine`` points the reference's ``Generator`` at this package's
``Decoder`` and ``KVPagePool`` and lets its ``PrefixCache`` take this package's paged
snapshots. These CPU tests run the reference's scheduler tick unchanged
(``Engine._continuous_tick``, src/helios/runtime/engine.py:197-214) with the model forward
replaced by a fake that acquires pages and advances lengths the way a tick does, so
admission, chunked prefill selection, sampling hand-off, completion, prefix-cache storage
and restore-by-aliasing are exercised on the host. The GPU test
(tests/test_gpu_reference_engine.py) runs the same engine with the real kernels.

Skipped when the reference package is not importable (set HELIOS_REFERENCE_SRC or
install it into baseline/_ref).
"""

from __future__ import annotations

import math

import pytest
import torch

from helios_b200.config import Qwen3Config
from helios_b200.decode import Decoder
from helios_b200.model import Qwen3Model
from helios_b200.paged_cache import KVPagePool, PagedKVBlockSnapshot, PagedKVCache

reference_engine = pytest.importorskip("helios_b200.reference_engine")
try:
    reference_engine.import_reference()
except reference_engine.ReferenceUnavailable as error:  # pragma: no cover - depends on the box
    pytest.skip(str(error), allow_module_level=True)

VOCAB = 64


def _tiny_model() -> Qwen3Model:
    cfg = Qwen3Config(vocab_size=VOCAB, context_length=4096, hidden_size=16, n_heads=2, n_layers=1, hidden_dim=32,
                      head_dim=8, n_kv_heads=1, dtype=torch.float32)
    torch.manual_seed(0)
    return Qwen3Model(cfg).eval()


def _advance(cache: PagedKVCache, count: int) -> None:
    pool = cache.pool
    missing = math.ceil((cache.length + count) / pool.page_size) - len(cache.pages)
    if missing > 0:
        cache.pages.extend(pool.acquire(missing))
    cache.length += count


def _next_logits(tokens: list[int]) -> torch.Tensor:
    """Fake forward: the next token is always (last token + 1) mod VOCAB."""
    out = torch.full((len(tokens), VOCAB), -1.0)
    for row, token in enumerate(tokens):
        out[row, (token + 1) % VOCAB] = 1.0
    return out


@pytest.fixture
def engine():
    from unittest.mock import patch

    with reference_engine.b200_path():
        eng = reference_engine.build_engine(_tiny_model(), kv_pages=32, max_batch_size=4, prefill_chunk_size=256,
                                            scheduler_thread=False)
        decoder = eng.generator.decoder
        ticks = {"packed": [], "decode": []}

        def packed(caches, chunks, *, logit_counts=None):
            ticks["packed"].append([len(c) for c in chunks])
            for cache, chunk in zip(caches, chunks):
                _advance(cache, len(chunk))
            counts = logit_counts or [1] * len(chunks)
            rows = [chunk[len(chunk) - n + i] for chunk, n in zip(chunks, counts) for i in range(n)]
            return _next_logits(rows)

        def decode(caches, tokens):
            ticks["decode"].append(len(tokens))
            for cache in caches:
                _advance(cache, 1)
            return _next_logits(tokens)

        with patch.object(decoder, "packed_caches", side_effect=packed), \
                patch.object(decoder, "decode_caches", side_effect=decode):
            eng.ticks = ticks
            yield eng
        eng.close()


def _finish(engine, *futures, limit=200):
    for _ in range(limit):
        if all(f.done() for f in futures):
            return [f.result(timeout=0) for f in futures]
        engine._continuous_tick(engine._scheduler)
    raise AssertionError("requests did not complete")


def test_engine_builds_this_packages_decoder_and_pool(engine):
    assert isinstance(engine.generator.decoder, Decoder)
    assert isinstance(engine.generator.decoder.page_pool, KVPagePool)
    assert engine.generator.decoder.page_pool.num_pages == 32


def test_continuous_ticks_admit_chunk_decode_and_complete(engine):
    from helios.runtime.types import Sampling

    greedy = Sampling(temperature=0, top_p=1, max_new_tokens=5)
    prompts = [[3] * 300, [7] * 40, [9] * 10]
    futures = [engine.enqueue(p, 0, greedy, request_id=f"r{i}") for i, p in enumerate(prompts)]
    results = _finish(engine, *futures)
    for prompt, result in zip(prompts, results):
        last = prompt[-1]
        assert result.output_ids == [(last + 1 + i) % VOCAB for i in range(5)]
        assert result.finish_reason == "length"
    # The first tick filled the 256-token budget (engine.py:343), splitting a prompt.
    assert sum(engine.ticks["packed"][0]) == 256
    assert engine.generator.decoder.page_pool.free_pages + len(engine.generator.prefix_cache.blocks()) == 32


def test_prefix_cache_stores_b200_snapshots_and_restores_them_by_aliasing(engine):
    from helios.runtime.types import Sampling

    greedy = Sampling(temperature=0, top_p=1, max_new_tokens=3)
    shared = list(range(1, 60)) * 9  # 531 tokens: two complete 256-token blocks
    first = engine.enqueue(shared + [5], 0, greedy, request_id="first")
    _finish(engine, first)
    blocks = engine.generator.prefix_cache._blocks
    assert len(blocks) == 2
    snapshots = [b.snapshot for b in blocks.values()]
    assert all(isinstance(s, PagedKVBlockSnapshot) for s in snapshots)
    assert engine.generator.prefix_cache.memory_bytes == 2 * snapshots[0].memory_bytes
    stored_pages = [p for s in snapshots for p in s.pages]

    restored = {}
    begin = engine.generator.decoder.begin_prefill

    def spy(*args, **kwargs):
        state = begin(*args, **kwargs)
        restored["pages"] = list(state.cache.pages)
        restored["offset"] = state.next_token_offset
        return state

    from unittest.mock import patch

    with patch.object(engine.generator.decoder, "begin_prefill", side_effect=spy):
        second = engine.enqueue(shared + [6, 7], 0, greedy, request_id="second")
        (result,) = _finish(engine, second)
    assert restored["offset"] == 512
    assert all(a is b for a, b in zip(restored["pages"], stored_pages))  # aliased, no copy
    assert result.prefix.hit_tokens == 512 and result.prefix.restored_tokens == 512
    assert result.output_ids == [7 + 1, 7 + 2, 7 + 3]


def test_begin_prefill_checks_match_the_reference(engine):
    from helios.runtime.types import Sampling

    decoder = engine.generator.decoder
    with pytest.raises(ValueError, match="KV-cache tokens"):
        decoder.begin_prefill([1] * 10, Sampling(max_new_tokens=20), max_total_tokens=16)
    free = decoder.page_pool.free_pages
    state = decoder.begin_prefill([1] * 10, Sampling(max_new_tokens=4), max_total_tokens=4096)
    assert state.next_token_offset == 0 and state.restored_tokens == 0 and state.cache.capacity == 14
    decoder.release_cache(state.cache)
    assert decoder.page_pool.free_pages == free
