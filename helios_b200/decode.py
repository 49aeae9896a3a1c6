"""Decoder entry points of the packed tick and the fused sampler.

Mirrors the reference's ``Decoder`` (src/helios/runtime/qwen3/decode.py:62-291):
``packed_caches`` (mixed / drafted ticks, :260-291) and ``decode_caches``
(decode-only ticks, :220-258) with the same arguments, checks and exceptions,
plus ``_sample`` (:457-473). Sampling runs in the fused CUDA sampler; a
caller-supplied ``uniforms`` tensor makes a draw deterministic, otherwise one
uniform per row is drawn on the device (no host synchronisation).

The rest of the reference decoder's surface that its ``Engine``, ``Generator`` and
warmup call (``begin_prefill`` :133-187, ``prefill_chunk`` :189-218, ``prefill``
:106-131, ``generate`` :68-104, ``decode`` :322-394, ``release_cache`` :403-408,
``_synchronize`` :435-439, ``device``) is here with the same arguments, results,
exceptions and timing semantics, so those callers run unchanged over this decoder
(``helios_b200.reference_engine`` swaps it in). Request caches are always paged:
there is no dense-KV path.

``sample_rows`` is the batched sampling of ``Engine._execute_batch``
(src/helios/runtime/engine.py:470-492): per-row temperature and top-p in one
launch instead of grouping rows by equal settings. ``sample_and_verify`` adds the
speculative verification of drafted rows (engine.py:488-520) on the device.
"""

from __future__ import annotations

import time
from collections.abc import Sequence
from dataclasses import dataclass
from itertools import accumulate

import torch

from helios_b200 import ops
from helios_b200.config import Sampling
from helios_b200.model import Qwen3Model
from helios_b200.paged_cache import KVPagePool, PackedBatchCache, PagedBatchCache, PagedKVCache


@dataclass
class PrefillState:
    """What ``begin_prefill`` hands the engine (decode.py:48-53)."""
    cache: PagedKVCache
    next_token_offset: int
    restore_seconds: float
    restored_tokens: int


@dataclass
class PrefillResult:
    """A whole-prompt prefill (decode.py:39-45): the last position's logits ``[1, V]``."""
    cache: PagedKVCache
    logits: torch.Tensor
    prefill_seconds: float
    restore_seconds: float
    restored_tokens: int


@dataclass
class DecodedTokens:
    """The decode loop's output (decode.py:56-62)."""
    first_token_at: float
    token_intervals: tuple[float, ...]
    output_ids: list[int]
    finish_reason: str
    inter_token_seconds: list[float]


@dataclass
class DecodeResult:
    """One request's generation (decode.py:25-36)."""
    first_token_at: float
    token_intervals: tuple[float, ...]
    output_ids: list[int]
    finish_reason: str
    prefill_seconds: float
    inter_token_seconds: list[float]
    restore_seconds: float
    restored_tokens: int
    cache: PagedKVCache


class Decoder:
    def __init__(self, model: Qwen3Model) -> None:
        self.model = model
        self.page_pool: KVPagePool | None = None
        self._paged_decode_batch: PagedBatchCache | None = None
        self._packed_batch: PackedBatchCache | None = None

    @property
    def device(self) -> torch.device:
        return next(self.model.parameters()).device

    # ---- single-request generation and admission (decode.py:68-218, :322-439)
    def generate(self, input_ids: list[int], eos_token_id: int, sampling: Sampling, *, max_total_tokens: int,
                 prefix_hit=None, request_id: str = "internal") -> DecodeResult:
        """Prefill then decode one request (decode.py:68-104); the cache stays open for the caller."""
        prefill = self.prefill(input_ids, sampling, max_total_tokens=max_total_tokens, prefix_hit=prefix_hit)
        try:
            decoded = self.decode(prefill, eos_token_id, sampling, request_id=request_id)
        except Exception:
            self.release_cache(prefill.cache)
            raise
        return DecodeResult(first_token_at=decoded.first_token_at, token_intervals=decoded.token_intervals,
                            output_ids=decoded.output_ids, finish_reason=decoded.finish_reason,
                            prefill_seconds=prefill.prefill_seconds, inter_token_seconds=decoded.inter_token_seconds,
                            restore_seconds=prefill.restore_seconds, restored_tokens=prefill.restored_tokens,
                            cache=prefill.cache)

    def prefill(self, input_ids: list[int], sampling: Sampling, *, max_total_tokens: int,
                prefix_hit=None) -> PrefillResult:
        """``begin_prefill`` plus one chunk of the rest of the prompt (decode.py:106-131)."""
        state = self.begin_prefill(input_ids, sampling, max_total_tokens=max_total_tokens, prefix_hit=prefix_hit)
        try:
            logits, seconds = self.prefill_chunk(state.cache, input_ids[state.next_token_offset:])
        except Exception:
            self.release_cache(state.cache)
            raise
        return PrefillResult(cache=state.cache, logits=logits, prefill_seconds=seconds,
                             restore_seconds=state.restore_seconds, restored_tokens=state.restored_tokens)

    def begin_prefill(self, input_ids: list[int], sampling: Sampling, *, max_total_tokens: int,
                      prefix_hit=None) -> PrefillState:
        """Open a paged request cache of ``len(input_ids) + max_new_tokens`` positions and alias the
        prefix-cache hit's pages into it (decode.py:133-187). ``prefix_hit`` is the reference's
        ``PrefixCacheHit`` (``blocks`` of ``tokens`` + ``snapshot``). On an exact full-prompt hit the
        last block is left out, so the final prompt token still runs and yields logits."""
        capacity = len(input_ids) + sampling.max_new_tokens
        if capacity > max_total_tokens:
            raise ValueError(f"Request needs {capacity:,} KV-cache tokens, but the profiled "
                             f"limit is {max_total_tokens:,}.")
        if self.page_pool is None:
            raise RuntimeError("The B200 decoder needs a KV page pool (Decoder.page_pool).")
        cache = PagedKVCache(self.page_pool, capacity)
        try:
            blocks = tuple(prefix_hit.blocks) if prefix_hit is not None else ()
            if blocks:
                if any(len(block.tokens) != block.snapshot.length for block in blocks):
                    raise ValueError("Prefix-cache token and KV block lengths do not match.")
                cached = [token for block in blocks for token in block.tokens]
                if len(cached) > len(input_ids):
                    raise ValueError("Prefix-cache hit is longer than the request prompt.")
                if list(input_ids[:len(cached)]) != cached:
                    raise ValueError("Prefix-cache hit does not match the request tokens.")
                if len(cached) == len(input_ids):
                    blocks = blocks[:-1]
            started = time.perf_counter()
            cache.restore_blocks(tuple(block.snapshot for block in blocks))
            restore_seconds = time.perf_counter() - started
            return PrefillState(cache=cache, next_token_offset=cache.length, restore_seconds=restore_seconds,
                                restored_tokens=cache.length)
        except Exception:
            self.release_cache(cache)
            raise

    def prefill_chunk(self, cache: PagedKVCache, input_ids_slice: Sequence[int] | torch.Tensor
                      ) -> tuple[torch.Tensor, float]:
        """Run one prompt chunk of one request; returns its last position's logits ``[1, V]`` and
        the synchronised wall time (decode.py:189-218). The chunk runs as a one-row packed tick,
        so only its last position goes through the lm_head."""
        if isinstance(input_ids_slice, torch.Tensor):
            tokens = input_ids_slice.to(dtype=torch.long)
            if tokens.ndim == 1:
                tokens = tokens.unsqueeze(0)
        else:
            tokens = torch.tensor(list(input_ids_slice), dtype=torch.long).unsqueeze(0)
        if tokens.ndim != 2 or tokens.shape[0] != 1 or tokens.shape[1] < 1:
            raise ValueError("Prefill chunks must contain at least one token with shape [1, tokens].")
        if self.model.training:
            self.model.eval()
        self._synchronize()
        started = time.perf_counter()
        logits = self._packed([cache], [tokens[0].tolist()], None, greedy=False)
        self._validate_forward_shapes(tokens[:, -1:], logits.unsqueeze(1))
        self._synchronize()
        return logits, time.perf_counter() - started

    def decode(self, prefill: PrefillResult, eos_token_id: int, sampling: Sampling, *,
               request_id: str = "internal") -> DecodedTokens:
        """Sample from the prefill logits, then decode one token per step until EOS or
        ``max_new_tokens`` (decode.py:322-394), timing each step between synchronisations."""
        first_token_at = last_token_at = None
        intervals: list[float] = []
        generated: list[int] = []
        inter_token_seconds: list[float] = []
        finish_reason = "length"
        logits, cache = prefill.logits, prefill.cache
        for index in range(sampling.max_new_tokens):
            next_token = self._sample(logits, sampling)
            token_id = int(next_token.item())
            sampled_at = time.perf_counter()
            if first_token_at is None:
                first_token_at = sampled_at
            if token_id == eos_token_id:
                finish_reason = "eos"
                break
            if last_token_at is not None:
                intervals.append(sampled_at - last_token_at)
            last_token_at = sampled_at
            generated.append(token_id)
            if index + 1 < sampling.max_new_tokens:
                self._synchronize()
                started = time.perf_counter()
                logits = self.decode_caches([cache], [token_id])
                self._validate_forward_shapes(next_token, logits.unsqueeze(1))
                self._synchronize()
                inter_token_seconds.append(time.perf_counter() - started)
        return DecodedTokens(first_token_at=first_token_at, token_intervals=tuple(intervals), output_ids=generated,
                             finish_reason=finish_reason, inter_token_seconds=inter_token_seconds)

    @staticmethod
    def release_cache(cache: PagedKVCache) -> None:
        """Return a request cache's pages to the pool (decode.py:403-408)."""
        cache.close()

    def _synchronize(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def _validate_forward_shapes(self, input_ids: torch.Tensor, logits: torch.Tensor) -> None:
        """Shape checks of one forward (decode.py:441-455), same messages."""
        if input_ids.ndim != 2 or input_ids.shape[0] != 1 or input_ids.shape[1] < 1:
            raise RuntimeError("Decoder input must have shape [1, tokens] with at least one token.")
        if input_ids.dtype != torch.long:
            raise RuntimeError("Decoder input token IDs must use torch.long.")
        expected = (1, 1, self.model.config.vocab_size)
        if tuple(logits.shape) != expected:
            raise RuntimeError(f"Decoder logits must have shape {expected}; received {tuple(logits.shape)}.")

    def decode_caches(self, caches: list[PagedKVCache], token_ids: list[int] | torch.Tensor) -> torch.Tensor:
        """Logits ``[B, V]`` of one decode step of every cache (decode.py:220-258).

        ``token_ids`` may also be a 1-D integer tensor on the pool's device (for instance the
        previous step's sampled ids): it is copied on the device, so a caller can queue the next
        step before it reads the previous step's ids back (the host half of a tick then overlaps
        the device half of the one before)."""
        return self._decode(caches, token_ids, greedy=False)

    def decode_caches_greedy(self, caches: list[PagedKVCache], token_ids: list[int] | torch.Tensor) -> torch.Tensor:
        """The temperature-0 next token of every cache (int64 ``[B]``): ``decode_caches`` followed
        by the argmax the reference samples greedy rows with (decode.py:458-460), with the argmax
        in the lm_head GEMM's epilogue so the logits are never written."""
        return self._decode(caches, token_ids, greedy=True)

    def _decode(self, caches: list[PagedKVCache], token_ids: list[int] | torch.Tensor, *,
                greedy: bool) -> torch.Tensor:
        if not caches or len(caches) != len(token_ids):
            raise ValueError("Every request cache needs exactly one pending token.")
        if isinstance(token_ids, torch.Tensor) and token_ids.device.type == "cpu":
            token_ids = token_ids.tolist()  # host ids take the list path
        on_device = isinstance(token_ids, torch.Tensor)
        pool_device = caches[0].pool.device
        if on_device and (token_ids.dim() != 1 or token_ids.device.type != pool_device.type
                          or (pool_device.index is not None and token_ids.device.index != pool_device.index)
                          or token_ids.dtype not in (torch.int32, torch.int64)):
            raise ValueError("Device token ids must be a 1-D integer tensor on the pool's device.")
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
                if on_device:
                    tokens = token_ids.to(torch.long).unsqueeze(1)
                else:
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
