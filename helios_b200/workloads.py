"""Model-level workloads beyond the bench's mixed tick.

    python -m helios_b200.workloads config4 [--steps N] [--no-share] [--sync]
    python -m helios_b200.workloads config4-decode [--ticks N] [--no-share] [--sync]

``config4``: BASELINE config 4 end to end on the Qwen3-4B architecture (random init, bf16,
seed 3). One request prefills the common 4096-token prefix through packed ticks and its 16
full pages are stored as prefix-cache blocks, keyed on the device (``DevicePrefixIndex``,
the reference's SHA-256 block chain). Then 128 requests, each the prefix plus its own tail
of U[256, 1024] tokens, are admitted: one device lookup finds each request's 16 stored
blocks and ``restore_blocks`` aliases their pages (no K/V bytes move). The tails are
prefilled through packed ticks of at most 2048 tokens (chunked, as the reference engine's
budget does), and every request then decodes ``steps`` (128) tokens with temperature 0.2
and top-p 0.95, one decode tick per step (CUDA-graph replay) sampled by kernel d, each
step's ids read back to the host (pipelined: while the GPU runs the next step, which takes
the ids on the device; ``--sync`` reads them before queueing it). Reports the restore cost (lookup + aliasing, and the
bytes it uploads), the tail prefill time and the decode tokens/s, each timed with CUDA
events.

``config4-decode``: the decode phase alone with random K/V standing in for the prefix and
tail prefill (the earlier measurement). ``--no-share`` switches off the shared-prefix
grouping (every row reads the prefix pages itself) for comparison. Each prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import sys
import time

import numpy as np
import torch

from helios_b200 import paged_cache
from helios_b200.config import Sampling, qwen3_4b_config
from helios_b200.decode import Decoder, sample_rows
from helios_b200.model import Qwen3Model
from helios_b200.paged_cache import KVPagePool, PagedKVCache

PREFIX_TOKENS, REQUESTS, TAIL = 4096, 128, (256, 1024)


def config2_batch(device: torch.device):
    """BASELINE config 2's inputs: one attention layer of the Qwen3-4B shape (32/8 heads,
    d=128), a 4096-page pool of N(0, 1/128) K/V (seed 1), 64 rows with contexts U[512, 8192]
    (the query token included) whose pages come from a random permutation of the pool, and
    one N(0, 1/128) query token per row. Returns ``(pool, batch, q, contexts)`` with the
    batch prepared (``prepare_packed([1] * 64)``)."""
    from helios_b200.config import Qwen3Config
    from helios_b200.paged_cache import PackedBatchCache

    cfg = Qwen3Config(n_layers=1, context_length=8192 + 64)
    g = torch.Generator().manual_seed(1)
    pool = KVPagePool(cfg, 4096, device=device)
    gen = torch.Generator(device=device).manual_seed(1)
    pool.storage.normal_(0.0, 1.0 / math.sqrt(128), generator=gen)
    contexts = torch.randint(512, 8193, (64,), generator=g).tolist()
    perm = torch.randperm(4096, generator=g).tolist()
    pool._free = list(reversed(perm))  # acquire() pops: pages come in permutation order
    caches = []
    for ctx in contexts:
        cache = PagedKVCache(pool, ctx)
        cache.pages.extend(pool.acquire(math.ceil((ctx - 1) / 256)))
        cache.length = ctx - 1
        caches.append(cache)
    batch = PackedBatchCache(caches)
    with torch.inference_mode():
        batch.prepare_packed([1] * 64)
    q = (torch.randn(64, 32, 128, generator=g) / math.sqrt(128)).to(torch.bfloat16).to(device)
    return pool, batch, q, contexts


def _cuda_timer(device):
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    return start, end


def decode_steps(tick, ids, steps: int, pipelined: bool = True) -> list[list[int]]:
    """Runs ``steps`` decode ticks from ``ids`` (a host list or a device tensor) through
    ``tick`` (token ids -> sampled ids on the device) and returns every step's sampled ids as
    read back to the host.

    Synchronous: each tick's ids come back (``.tolist``) before the next tick is queued, as the
    reference engine's loop does (src/helios/runtime/engine.py:406-530). Pipelined: the next tick
    takes the sampled ids on the device and is queued first; each step's ids are copied to pinned
    memory and read while the GPU runs the step after it, so the host half of a tick (page
    bookkeeping, the descriptor, tick packing) overlaps the device half of the one before. Both
    sample the same ids."""
    out: list[list[int]] = []
    if not pipelined:
        for _ in range(steps):
            ids = tick(ids).tolist()
            out.append(ids)
        return out
    host, done = None, [torch.cuda.Event(), torch.cuda.Event()]
    for step in range(steps):
        ids = tick(ids)
        if host is None:
            host = [torch.empty(ids.numel(), dtype=ids.dtype, pin_memory=True) for _ in range(2)]
        host[step & 1].copy_(ids, non_blocking=True)
        done[step & 1].record()
        if step:
            done[(step - 1) & 1].synchronize()
            out.append(host[(step - 1) & 1].tolist())
    if steps:
        done[(steps - 1) & 1].synchronize()
        out.append(host[(steps - 1) & 1].tolist())
    return out


def config4(steps: int = 128, share: bool = True, device: torch.device | None = None, seed: int = 3,
            warmup: int = 3, pipelined: bool = True) -> dict:
    """BASELINE config 4 as specified (see the module docstring); returns its measurements."""
    from helios_b200.prefix_index import DevicePrefixIndex

    device = device or torch.device("cuda", torch.cuda.current_device())
    cfg = qwen3_4b_config()
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen3Model(cfg).eval()
    decoder = Decoder(model)
    g = torch.Generator().manual_seed(seed)
    prefix = torch.randint(0, cfg.vocab_size, (PREFIX_TOKENS,), generator=g).tolist()
    tails = torch.randint(TAIL[0], TAIL[1] + 1, (REQUESTS,), generator=g).tolist()
    prompts = [prefix + torch.randint(0, cfg.vocab_size, (t,), generator=g).tolist() for t in tails]
    prefix_pages = PREFIX_TOKENS // 256
    total_steps = warmup + steps
    pages = prefix_pages + 1 + sum(math.ceil((len(p) + total_steps + 1) / 256) - prefix_pages for p in prompts) + 8
    pool = decoder.page_pool = KVPagePool(cfg, pages, device=device)
    saved = paged_cache.MIN_SHARED_PAGES
    if not share:
        paged_cache.MIN_SHARED_PAGES = 1 << 30
    try:
        with torch.inference_mode():
            # The first request: the prefix prefilled in 2048-token packed ticks, its full
            # blocks stored and keyed on the device.
            donor = PagedKVCache(pool, PREFIX_TOKENS + 1)
            for at in range(0, PREFIX_TOKENS, 2048):
                decoder.packed_caches([donor], [prefix[at:at + 2048]])
            blocks = [donor.snapshot_block(b * 256, (b + 1) * 256) for b in range(prefix_pages)]
            index = DevicePrefixIndex(4 * prefix_pages, 256, device)
            from helios_b200.prefix_index import hash_token_blocks

            keys = hash_token_blocks([prefix], 256, device)[0]
            index.add(keys, list(range(prefix_pages)))
            donor.close()
            torch.cuda.synchronize(device)

            # The prompts as a tokenizer hands them over (int32 arrays): the lookup then needs
            # no per-token conversion of Python ints on the host.
            arrays = [np.asarray(p, dtype=np.int32) for p in prompts]
            index.lookup(arrays)  # first call: sizes the reused pinned staging, loads the kernels; untimed
            torch.cuda.synchronize(device)
            # Admission: one device lookup for all 128 prompts, then aliasing restores.
            start, end = _cuda_timer(device)
            t0 = time.perf_counter()
            start.record()
            hits = index.lookup(arrays)
            caches = []
            for prompt, (_, values) in zip(prompts, hits):
                cache = PagedKVCache(pool, len(prompt) + total_steps + 1)
                cache.restore_blocks([blocks[v] for v in values])
                caches.append(cache)
            end.record()
            torch.cuda.synchronize(device)
            restore_wall = time.perf_counter() - t0
            restore_gpu = start.elapsed_time(end) / 1e3
            restored = [c.length for c in caches]

            # Tails: packed ticks of at most 2048 prompt tokens, rows chunked across ticks. Every
            # tail tick has its own shape, so they run eagerly (a graph would be captured per
            # tick and never replayed); the decode steps below replay graphs.
            model._graphs = None
            offsets = list(restored)
            ticks = 0
            first_logits = {}
            start, end = _cuda_timer(device)
            start.record()
            pending = list(range(REQUESTS))
            while pending:
                budget, rows, chunks = 2048, [], []
                for r in list(pending):
                    if budget == 0:
                        break
                    n = min(budget, len(prompts[r]) - offsets[r])
                    rows.append(r)
                    chunks.append(prompts[r][offsets[r]:offsets[r] + n])
                    offsets[r] += n
                    budget -= n
                    if offsets[r] == len(prompts[r]):
                        pending.remove(r)
                logits = decoder.packed_caches([caches[r] for r in rows], chunks)
                for i, r in enumerate(rows):
                    if offsets[r] == len(prompts[r]):
                        first_logits[r] = logits[i].clone()  # graph outputs are reused by later replays
                ticks += 1
            heads = torch.stack([first_logits[r] for r in range(REQUESTS)])
            end.record()
            torch.cuda.synchronize(device)
            prefill_seconds = start.elapsed_time(end) / 1e3
            tail_tokens = sum(len(p) for p in prompts) - sum(restored)

            model.enable_cuda_graphs()
            samplings = [Sampling(temperature=0.2, top_p=0.95, max_new_tokens=total_steps + 1)] * REQUESTS
            sample_gen = torch.Generator(device=device).manual_seed(seed)
            ids = sample_rows(heads, samplings, generator=sample_gen).tolist()

            def tick(token_ids):
                out = decoder.decode_caches(caches, token_ids)
                return sample_rows(out, samplings, generator=sample_gen)

            for _ in range(warmup):  # eager tick, graph capture, first replay
                ids = tick(ids).tolist()
            torch.cuda.synchronize(device)
            start, end = _cuda_timer(device)
            start.record()
            decode_steps(tick, ids, steps, pipelined)
            end.record()
            torch.cuda.synchronize(device)
            decode_seconds = start.elapsed_time(end) / 1e3
    finally:
        paged_cache.MIN_SHARED_PAGES = saved
    return {
        "workload": "BASELINE config 4: 128 requests = shared 4096-token prefix (16 blocks, device-keyed) + own "
                    "tail U[256,1024]; tails prefilled in packed ticks of <= 2048 tokens; 128 decode steps at "
                    "T=0.2 top-p 0.95, seed 3",
        "restore": {"blocks_per_request": prefix_pages, "restored_tokens_per_request": min(restored),
                    "us_gpu": round(restore_gpu * 1e6, 1), "us_wall": round(restore_wall * 1e6, 1),
                    "kv_bytes_moved": 0,
                    "metadata_bytes": REQUESTS * prefix_pages * 4,
                    "what": "one hb_hash_token_blocks + hb_prefix_index_lookup over the 128 prompts (int32 "
                            "arrays), then page aliasing; the restored page ids reach the device arena with the "
                            "next tick's descriptor (4 bytes per page)"},
        "tail_prefill": {"tokens": tail_tokens, "ticks": ticks, "seconds": round(prefill_seconds, 4),
                         "tokens_per_s": round(tail_tokens / prefill_seconds, 1)},
        "decode": {"steps": steps, "ms_per_step": round(1e3 * decode_seconds / steps, 3),
                   "tokens_per_s": round(REQUESTS * steps / decode_seconds, 1),
                   "timing": "CUDA events around the decode steps; each step's sampled ids read back to the host "
                             + ("while the GPU runs the next step (the next tick takes the ids on the device)"
                                if pipelined else "before the next step is queued")},
        "shared_prefix_grouping": share,
    }


def config4_decode(ticks: int, share: bool, warmup: int = 3, pipelined: bool = True) -> dict:
    device = torch.device("cuda", 0)
    cfg = qwen3_4b_config()
    torch.manual_seed(3)
    with torch.device(device):
        model = Qwen3Model(cfg).eval()
    model.enable_cuda_graphs()
    g = torch.Generator().manual_seed(3)
    tails = torch.randint(TAIL[0], TAIL[1] + 1, (REQUESTS,), generator=g).tolist()
    steps = warmup + ticks + 1
    prefix_pages = PREFIX_TOKENS // 256
    pages = prefix_pages + sum(math.ceil((PREFIX_TOKENS + t + steps) / 256) - prefix_pages for t in tails) + 8
    pool = KVPagePool(cfg, pages, device=device)
    gen = torch.Generator(device=device).manual_seed(3)
    for layer in range(cfg.n_layers):
        pool.storage[layer].normal_(0.0, 0.3, generator=gen)
    prefix = PagedKVCache(pool, PREFIX_TOKENS)
    prefix.pages.extend(pool.acquire(prefix_pages))
    prefix.length = PREFIX_TOKENS
    block = prefix.snapshot_block(0, PREFIX_TOKENS)
    caches = []
    for tail in tails:
        cache = PagedKVCache(pool, PREFIX_TOKENS + tail + steps + 8)
        cache.restore_blocks([block])  # the shared pages, aliased
        cache.pages.extend(pool.acquire(math.ceil((PREFIX_TOKENS + tail) / 256) - prefix_pages))
        cache.length = PREFIX_TOKENS + tail
        caches.append(cache)
    decoder = Decoder(model)
    decoder.page_pool = pool
    samplings = [Sampling(temperature=0.2, top_p=0.95, max_new_tokens=steps)] * REQUESTS
    ids = torch.randint(0, cfg.vocab_size, (REQUESTS,), generator=g).tolist()
    sample_gen = torch.Generator(device=device).manual_seed(3)
    saved = paged_cache.MIN_SHARED_PAGES
    if not share:
        paged_cache.MIN_SHARED_PAGES = 1 << 30
    try:
        def tick(token_ids):
            logits = decoder.decode_caches(caches, token_ids)
            return sample_rows(logits, samplings, generator=sample_gen)

        for _ in range(warmup):
            ids = tick(ids).tolist()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()

        def marked(token_ids):
            torch.cuda.nvtx.range_push("tick")  # lets a profiler select exactly the timed ticks
            try:
                return tick(token_ids)
            finally:
                torch.cuda.nvtx.range_pop()

        decode_steps(marked, ids, ticks, pipelined)
        end.record()
        torch.cuda.synchronize()
    finally:
        paged_cache.MIN_SHARED_PAGES = saved
    ms = start.elapsed_time(end) / ticks
    return {"workload": "BASELINE config 4 decode: 128 requests, 4096-token shared prefix, tails U[256,1024], "
                        "T=0.2 top-p 0.95", "model": "Qwen3-4B architecture, random init", "dtype": "bf16",
            "shared_prefix_grouping": share, "ticks": ticks, "ms_per_tick": round(ms, 3),
            "tokens_per_s": round(REQUESTS / (ms / 1e3), 1),
            "timing": "CUDA events around the ticks, each tick's ids read back to the host "
                      + ("while the GPU runs the next tick" if pipelined else "before the next tick is queued")}


def main(argv: list[str]) -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("workload", choices=("config4", "config4-decode"))
    parser.add_argument("--ticks", type=int, default=16)
    parser.add_argument("--steps", type=int, default=128)
    parser.add_argument("--no-share", action="store_true")
    parser.add_argument("--sync", action="store_true",
                        help="read each step's ids back before queueing the next step (no pipelining)")
    args = parser.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("the workloads need a CUDA device")
    if args.workload == "config4":
        print(json.dumps(config4(args.steps, not args.no_share, pipelined=not args.sync)), flush=True)
    else:
        print(json.dumps(config4_decode(args.ticks, not args.no_share, pipelined=not args.sync)), flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])
