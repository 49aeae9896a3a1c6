"""continuous-batching load on the reference's Engine over the B200 path.

    python -m helios_b200.load [--rates 16,32,64] [--requests 2048] [--cap-seconds 60]
    torchrun --nproc-per-node N -m helios_b200.load ...     (one replica per GPU)

Requests: Poisson arrivals at ``rate`` per GPU, prompt lengths lognormal (median 600,
sigma 0.8) clipped to [16, 8192], ``max_new_tokens`` uniform in [64, 512], token ids
uniform, the reference's default sampling (temperature 0.2, top-p 0.95). Each replica (one
process per GPU) runs one reference ``Engine`` (its scheduler thread, admission, tick
selection under a 2048-token budget, prefix cache, sampling and completion, all
unchanged, src/helios/runtime/engine.py:184-530) with max batch 128, whose decoder, page
pool and model are this package's (``helios_b200.reference_engine``). The global request
stream is sharded round-robin (``replicas.shard``), so each replica sees Poisson arrivals
at ``rate``. A feeder thread enqueues each request at its arrival time
(``Engine.enqueue``, engine.py:184-195).

Reported per rate: aggregate output tokens/s (all replicas' generated tokens over the
slowest replica's span from its first arrival to its last completion), p50 and p90
time to first token over all requests (the reference's ``first_token_seconds``: from
enqueue to the first sampled token), and requests and tokens served.
"""

from __future__ import annotations

import argparse
import json
import math
import statistics
import threading
import time

import numpy as np
import torch

PROMPT_MEDIAN, PROMPT_SIGMA, PROMPT_CLIP = 600, 0.8, (16, 8192)
MAX_TOKENS = (64, 512)
TICK_BUDGET, MAX_BATCH = 2048, 128
EOS = 0  # prompts draw ids from [1, vocab); an EOS the model samples ends its request early


def _log(text: str) -> None:
    import sys

    print(f"[load] {text}", file=sys.stderr, flush=True)


def make_requests(n: int, vocab: int, seed: int) -> list[tuple[list[int], int]]:
    """``n`` (prompt ids, max_new_tokens) pairs with BASELINE config 5's distributions."""
    rng = np.random.default_rng(seed)
    lengths = np.clip(np.round(rng.lognormal(math.log(PROMPT_MEDIAN), PROMPT_SIGMA, n)), *PROMPT_CLIP).astype(int)
    limits = rng.integers(MAX_TOKENS[0], MAX_TOKENS[1] + 1, n)
    return [(rng.integers(1, vocab, int(length)).tolist(), int(limit)) for length, limit in zip(lengths, limits)]


def arrival_times(n: int, rate: float, seed: int) -> np.ndarray:
    """Poisson process: cumulative exponential gaps of mean ``1/rate`` seconds."""
    rng = np.random.default_rng(seed + 1)
    return np.cumsum(rng.exponential(1.0 / rate, n))


def kv_pages_for(device: torch.device, config, fraction: float = 0.6) -> int:
    free, _ = torch.cuda.mem_get_info(device)
    page_bytes = config.n_layers * 2 * config.n_kv_heads * config.head_dim * 2 * 256
    return int(free * fraction // page_bytes)


def run_replica(engine, requests: list[tuple[list[int], int]], arrivals: np.ndarray) -> dict:
    """Feed ``requests`` to ``engine`` at ``arrivals`` (seconds from now) and wait for all."""
    from helios.runtime.types import Sampling

    futures: list = [None] * len(requests)
    start = time.perf_counter()

    def feed():
        for i, ((prompt, limit), at) in enumerate(zip(requests, arrivals)):
            delay = start + at - time.perf_counter()
            if delay > 0:
                time.sleep(delay)
            futures[i] = engine.enqueue(prompt, EOS, Sampling(max_new_tokens=limit), request_id=f"load-{i}")

    feeder = threading.Thread(target=feed, name="load-feeder", daemon=True)
    feeder.start()
    feeder.join()
    results = [f.result() for f in futures]
    done = time.perf_counter()
    tokens = sum(len(r.output_ids) for r in results)
    return {"requests": len(results), "output_tokens": tokens, "span_s": done - start,
            "ttft_s": [r.first_token_seconds for r in results if r.first_token_seconds is not None],
            "prompt_tokens": sum(len(p) for p, _ in requests)}


def build(device: torch.device, seed: int):
    """A random-init Qwen3-4B B200 model and a reference Engine over it (scheduler thread on)."""
    from helios_b200 import reference_engine
    from helios_b200.config import qwen3_4b_config
    from helios_b200.model import Qwen3Model

    cfg = qwen3_4b_config()
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen3Model(cfg).eval()
    context = reference_engine.b200_path()
    context.__enter__()
    engine = reference_engine.build_engine(model, kv_pages=kv_pages_for(device, cfg), max_batch_size=MAX_BATCH,
                                           prefill_chunk_size=TICK_BUDGET, max_queue_size=1 << 16,
                                           batch_wait_ms=2.0)
    return engine, context


def measure(rate: float, total_requests: int, *, seed: int = 5, device: torch.device | None = None,
            engine=None, warmup_requests: int = 16) -> dict:
    """One load point on this process's replica; all ranks must call it together."""
    from helios_b200 import replicas
    from helios_b200.config import qwen3_4b_config

    rank, size, local = replicas.world()
    device = device or torch.device("cuda", local)
    own_engine = engine is None
    context = None
    if own_engine:
        engine, context = build(device, seed)
    try:
        vocab = qwen3_4b_config().vocab_size
        if warmup_requests:  # kernels, library handles and allocator blocks, outside the measurement
            warm = make_requests(warmup_requests, vocab, seed + 100 + rank)
            run_replica(engine, warm, np.zeros(len(warm)))
        _log(f"rank {rank}: warm-up done")
        requests = make_requests(total_requests, vocab, seed)
        arrivals = arrival_times(total_requests, rate * size, seed)
        mine = replicas.shard(list(range(total_requests)), rank, size)
        replicas.barrier(device)
        out = run_replica(engine, [requests[i] for i in mine], arrivals[mine] - (arrivals[mine][0] if mine else 0))
        _log(f"rank {rank}: {out['requests']} requests, {out['output_tokens']} tokens in {out['span_s']:.2f} s")
    finally:
        if own_engine:
            engine.close()
            context.__exit__(None, None, None)
    gathered = replicas.gather_objects(out, device)
    if rank != 0:
        return {}
    span = max(r["span_s"] for r in gathered)
    ttft = sorted(t for r in gathered for t in r["ttft_s"])
    tokens = sum(r["output_tokens"] for r in gathered)
    return {"rate_per_gpu": rate, "replicas": size, "requests": sum(r["requests"] for r in gathered),
            "output_tokens": tokens, "prompt_tokens": sum(r["prompt_tokens"] for r in gathered),
            "span_s": round(span, 3), "tokens_per_s": round(tokens / span, 1),
            "ttft_p50_ms": round(1e3 * statistics.median(ttft), 1) if ttft else None,
            "ttft_p90_ms": round(1e3 * ttft[int(0.9 * (len(ttft) - 1))], 1) if ttft else None}


def main() -> None:
    from helios_b200 import replicas

    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--rates", default="16,32,64", help="arrival rates per GPU (requests/s), comma-separated")
    parser.add_argument("--requests", type=int, default=2048, help="requests per rate, over all replicas")
    parser.add_argument("--cap-seconds", type=float, default=60.0,
                        help="at most this many seconds of arrivals per rate (fewer requests at low rates)")
    parser.add_argument("--seed", type=int, default=5)
    args = parser.parse_args()
    rank, size, local = replicas.world()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    replicas.init("nccl" if size > 1 else "gloo")
    engine, context = build(device, args.seed)
    try:
        for rate in (float(r) for r in args.rates.split(",")):
            n = int(min(args.requests, rate * size * args.cap_seconds))
            point = measure(rate, n, seed=args.seed, device=device, engine=engine)
            if rank == 0:
                print(json.dumps({"workload": "BASELINE config 5", **point}), flush=True)
    finally:
        engine.close()
        context.__exit__(None, None, None)
        replicas.shutdown()


if __name__ == "__main__":
    main()
