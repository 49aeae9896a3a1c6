"""Decoder entry points of the packed tick and the fused sampler.

Mirrors the reference's ``Decoder`` (src/helios/runtime/qwen3/decode.py:62-291):
``packed_caches`` (mixed / drafted ticks, :260-291) and ``decode_caches``
(decode-only ticks, :220-258) with the same arguments, checks and exceptions,
plus ``_sample`` (:457-473). Sampling runs in the fused CUDA sampler; a
caller-supplied ``uniforms`` tensor makes a draw deterministic, otherwise one
uniform per row is drawn on the device (no host synchronisation).

``sample_rows`` is the batched sampling of ``Engine._execute_batch``
(src/helios/runtime/engine.py:470-492): per-row temperature and top-p in one
launch instead of grouping rows by equal settings. ``sample_and_verify`` adds the
speculative verification of drafted rows (engine.py:488-520) on the device.
"""

from __future__ import annotations

from collections.abc import Sequence
from itertools import accumulate

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
        """Logits ``[B, V]`` of one decode step of every cache (decode.py:220-258)."""
        return self._decode(caches, token_ids, greedy=False)

    def decode_caches_greedy(self, caches: list[PagedKVCache], token_ids: list[int]) -> torch.Tensor:
        """The temperature-0 next token of every cache (int64 ``[B]``): ``decode_caches`` followed
        by the argmax the reference samples greedy rows with (decode.py:458-460), with the argmax
        in the lm_head GEMM's epilogue so the logits are never written."""
        return self._decode(caches, token_ids, greedy=True)

    def _decode(self, caches: list[PagedKVCache], token_ids: list[int], *, greedy: bool) -> torch.Tensor:
        if not caches or len(caches) != len(token_ids):
            raise ValueError("Every request cache needs exactly one pending token.")
        if any(not isinstance(cache, PagedKVCache) or cache.pool is not caches[0].pool for cache in caches):
            raise ValueError("Paged decode caches must share one pool.")
        if len({id(cache) for cache in caches}) != len(caches):
            raise ValueError("Paged batches require distinct request caches.")
        if self.model.training:  # a recursive eval() walks ~500 modules: about 1 ms per tick
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
                if greedy:
                    return self.model.greedy_ids(tokens, batch, cache_slots=slots)
                return self.model(tokens, cache=batch, cache_slots=slots)[:, -1, :]
            finally:
                batch.caches = ()

    def packed_caches(self, caches: list[PagedKVCache], chunks: list[list[int]], *,
                      logit_counts: list[int] | None = None) -> torch.Tensor:
        """Logits ``[sum(logit_counts), V]`` of one packed mixed tick (decode.py:260-291)."""
        return self._packed(caches, chunks, logit_counts, greedy=False)

    def packed_caches_greedy(self, caches: list[PagedKVCache], chunks: list[list[int]], *,
                             logit_counts: list[int] | None = None) -> torch.Tensor:
        """Temperature-0 token ids (int64 ``[sum(logit_counts)]``) of the logit rows
        ``packed_caches`` returns, with the argmax in the lm_head GEMM's epilogue."""
        return self._packed(caches, chunks, logit_counts, greedy=True)

    def _packed(self, caches: list[PagedKVCache], chunks: list[list[int]], logit_counts: list[int] | None, *,
                greedy: bool) -> torch.Tensor:
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
                if greedy:
                    return self.model.greedy_ids(tokens, batch)
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
    if device.type == "cuda":
        # From pinned memory the upload queues behind the tick instead of waiting for it.
        settings = settings.pin_memory().to(device, non_blocking=True)
    else:
        settings = settings.to(device)
    if uniforms is None:
        uniforms = torch.rand(rows, dtype=torch.float32, device=device, generator=generator)
    elif uniforms.dtype != torch.float32 or uniforms.device != device:
        uniforms = uniforms.to(device=device, dtype=torch.float32)
    if logits.dtype != torch.bfloat16:
        logits = logits.to(torch.bfloat16)
    return ops.sample(logits, settings[:, 0].contiguous(), settings[:, 1].contiguous(), uniforms.contiguous())


_GREEDY = Sampling(max_new_tokens=1, temperature=0.0, top_p=1.0)


def sample_and_verify(logits: torch.Tensor, chunks: Sequence[Sequence[int]], logit_counts: Sequence[int],
                      samplings: Sequence[Sampling], *, caches: Sequence[PagedKVCache] | None = None,
                      cache_lengths: Sequence[int] | None = None,
                      uniforms: torch.Tensor | None = None) -> list[list[int]]:
    """Tokens each row of a packed tick emits, with speculative drafts verified on the device.

    ``logits [sum(logit_counts), V]`` come from ``Decoder.packed_caches(..., logit_counts=...)``.
    As in Engine._execute_batch (src/helios/runtime/engine.py:466-520): every row's head
    (its first logit row) is drawn with the row's sampling; the other logit rows of a
    drafted row get their greedy ids (drafts are only proposed for temperature-0 requests,
    engine.py:380); a drafted row accepts the longest prefix of its drafts (its chunk after
    the pending token) matching those ids and emits ids 0 .. accepted. Sampling,
    verification and the emitted tokens stay on the device; one transfer brings back the
    accepted counts and tokens. With ``caches`` and their ``cache_lengths`` from before the
    tick, each drafted row's cache is truncated to ``length + 1 + accepted`` (engine.py:515).
    """
    rows = len(chunks)
    if len(logit_counts) != rows or len(samplings) != rows:
        raise ValueError("Each chunk needs its logit count and sampling settings.")
    if any(not 1 <= lc <= len(chunk) for chunk, lc in zip(chunks, logit_counts, strict=True)):
        raise ValueError("Logit rows must be 1 through each chunk length.")
    starts = list(accumulate(logit_counts, initial=0))
    if logits.shape[0] != starts[-1]:
        raise ValueError("Logits must hold one row per logit count.")
    per_row = []
    for sampling, lc in zip(samplings, logit_counts, strict=True):
        per_row.append(sampling)
        per_row.extend([_GREEDY] * (lc - 1))
    device = logits.device
    predictions = sample_rows(logits, per_row, uniforms=uniforms)
    # One pinned upload of the draft tokens, chunk bounds and logit offsets (int64), queued
    # behind the tick.
    cu_host = list(accumulate((len(c) for c in chunks), initial=0))
    packed = torch.tensor([t for chunk in chunks for t in chunk] + cu_host + starts, dtype=torch.long)
    if device.type == "cuda":
        packed = packed.pin_memory().to(device, non_blocking=True)
    else:
        packed = packed.to(device)
    n_tok = cu_host[-1]
    tokens = packed[:n_tok]
    cu = packed[n_tok:n_tok + rows + 1].int()
    offsets = packed[n_tok + rows + 1:].int()
    accepted, emitted = ops.verify_drafts(tokens, cu, offsets, predictions)
    host = torch.cat([accepted.long(), emitted]).cpu().tolist()  # the tick's one device->host transfer
    counts, flat = host[:rows], host[rows:]
    out = []
    for row in range(rows):
        out.append(flat[starts[row]: starts[row] + counts[row] + 1])
        if caches is not None and logit_counts[row] > 1:
            if cache_lengths is None:
                raise ValueError("Truncating drafted rows needs their cache lengths before the tick.")
            caches[row].truncate(cache_lengths[row] + 1 + counts[row])
    return out
