"""Model-level workloads beyond the bench's mixed tick.

    python -m helios_b200.workloads config4 [--ticks N] [--no-share]

``config4``: BASELINE config 4's decode phase on the Qwen3-4B architecture (random init,
bf16). 128 requests share a 4096-token prefix (16 pages stored once and restored into every
request by page aliasing), each with its own tail of U[256, 1024] tokens. Random K/V stand in
for the prefix and tail prefill. Every tick decodes one token per request through
``Decoder.decode_caches`` (CUDA-graph replay of the device half), then samples them with
temperature 0.2 and top-p 0.95 (kernel d). The timed ticks are bracketed by CUDA events.
``--no-share`` switches off the shared-prefix grouping (every row reads the prefix pages
itself) for comparison. Prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import sys

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


def config4(ticks: int, share: bool, warmup: int = 3) -> dict:
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
        out = None
        for _ in range(ticks):
            torch.cuda.nvtx.range_push("tick")  # lets a profiler select exactly the timed ticks
            out = tick(ids if out is None else out.tolist())
            torch.cuda.nvtx.range_pop()
        end.record()
        torch.cuda.synchronize()
    finally:
        paged_cache.MIN_SHARED_PAGES = saved
    ms = start.elapsed_time(end) / ticks
    return {"workload": "BASELINE config 4 decode: 128 requests, 4096-token shared prefix, tails U[256,1024], "
                        "T=0.2 top-p 0.95", "model": "Qwen3-4B architecture, random init", "dtype": "bf16",
            "shared_prefix_grouping": share, "ticks": ticks, "ms_per_tick": round(ms, 3),
            "tokens_per_s": round(REQUESTS / (ms / 1e3), 1),
            "timing": "CUDA events around the ticks, each tick's ids read back to the host (.tolist)"}


def main(argv: list[str]) -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("workload", choices=("config4",))
    parser.add_argument("--ticks", type=int, default=16)
    parser.add_argument("--no-share", action="store_true")
    args = parser.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("the workloads need a CUDA device")
    print(json.dumps(config4(args.ticks, not args.no_share)), flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])
