"""Decoder entry points of the packed tick and the fused sampler.

Mirrors the reference's ``Decoder`` (src/helios/runtime/qwen3/decode.py:62-291):
``packed_caches`` (mixed / drafted ticks, :260-291) and ``decode_caches``
(decode-only ticks, :220-258) with the same arguments, checks and exceptions,
plus ``_sample`` (:457-473). Sampling runs in the fused CUDA sampler; a
caller-supplied ``uniforms`` tensor makes a draw deterministic, otherwise one
uniform per row is drawn on the device (no host synchronisation).

``sample_rows`` is the batched sampling of ``Engine._execute_batch``
(src/helios/runtime/engine.py:470-492): per-row temperature and top-p in one
launch instead of grouping rows by equal settings.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from helios_b200 import ops
from helios_b200.config import Sampling
from helios_b200.model import Qwen3Model
from helios_b200.paged_cache import KVPagePool, PackedBatchCache, PagedBatchCache, PagedKVCache


class Decoder:
    def __init__(self, model: Qwen3Model) -> None:
        self.model = model
        self.page_pool: KVPagePool | None = None
        self._paged_decode_batch: PagedBatchCache | None = None
        self._packed_batch: PackedBatchCache | None = None

    @property
    def device(self) -> torch.device:
        return next(self.model.parameters()).device

    def decode_caches(self, caches: list[PagedKVCache], token_ids: list[int]) -> torch.Tensor:
        if not caches or len(caches) != len(token_ids):
            raise ValueError("Every request cache needs exactly one pending token.")
        if any(not isinstance(cache, PagedKVCache) or cache.pool is not caches[0].pool for cache in caches):
            raise ValueError("Paged decode caches must share one pool.")
        if len({id(cache) for cache in caches}) != len(caches):
            raise ValueError("Paged batches require distinct request caches.")
        self.model.eval()
        with torch.inference_mode():
            batch = self._paged_decode_batch
            if batch is None or batch.pool is not caches[0].pool:
                batch = self._paged_decode_batch = PagedBatchCache(caches)
            batch.caches = tuple(caches)
            batch.batch_size = len(caches)
            try:
                tokens = batch.metadata("token_ids", list(token_ids), torch.long).unsqueeze(1)
                batch.prepare(1)
                slots = tuple(range(len(caches)))
                return self.model(tokens, cache=batch, cache_slots=slots)[:, -1, :]
            finally:
                batch.caches = ()

    def packed_caches(self, caches: list[PagedKVCache], chunks: list[list[int]], *,
                      logit_counts: list[int] | None = None) -> torch.Tensor:
        if not caches or len(caches) != len(chunks) or any(not chunk for chunk in chunks):
            raise ValueError("Each packed cache needs a nonempty token chunk.")
        if len({id(cache) for cache in caches}) != len(caches) or any(
                cache.pool is not caches[0].pool for cache in caches):
            raise ValueError("Packed caches must be distinct and share a pool.")
        with torch.inference_mode():
            batch = self._packed_batch
            if batch is None or batch.pool is not caches[0].pool:
                batch = self._packed_batch = PackedBatchCache(caches)
            batch.caches, batch.batch_size = tuple(caches), len(caches)
            try:
                tokens = batch.metadata("token_ids", [t for chunk in chunks for t in chunk], torch.long).unsqueeze(0)
                batch.prepare_packed([len(chunk) for chunk in chunks], logit_counts)
                return self.model(tokens, cache=batch)
            finally:
                batch.caches = ()

    @staticmethod
    def _sample(logits: torch.Tensor, sampling: Sampling, uniforms: torch.Tensor | None = None) -> torch.Tensor:
        """``[rows, V]`` -> ``[rows, 1]`` token ids, as decode.py:457-473 returns."""
        rows = logits.reshape(-1, logits.shape[-1])
        return sample_rows(rows, [sampling] * rows.shape[0], uniforms=uniforms).unsqueeze(-1)


def sample_rows(logits: torch.Tensor, samplings: Sequence[Sampling], *, uniforms: torch.Tensor | None = None,
                generator: torch.Generator | None = None) -> torch.Tensor:
    """One token id per logit row with per-row temperature / top-p (kernel d)."""
    rows = logits.shape[0]
    if len(samplings) != rows:
        raise ValueError("Each logit row needs its sampling settings.")
    device = logits.device
    settings = torch.tensor([[s.temperature, s.top_p] for s in samplings], dtype=torch.float32)
    settings = settings.to(device)
    if uniforms is None:
        uniforms = torch.rand(rows, dtype=torch.float32, device=device, generator=generator)
    elif uniforms.dtype != torch.float32 or uniforms.device != device:
        uniforms = uniforms.to(device=device, dtype=torch.float32)
    if logits.dtype != torch.bfloat16:
        logits = logits.to(torch.bfloat16)
    return ops.sample(logits, settings[:, 0].contiguous(), settings[:, 1].contiguous(), uniforms.contiguous())
