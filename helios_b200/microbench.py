"""Kernel microbenchmarks at the BASELINE config-3 tick shapes, timed from CUDA-graph replays.

    python -m helios_b200.microbench [norm_rope] [swiglu] [add_rmsnorm] [prefill] [decode] [mixed[:N]] [prefix_decode] [sample]
                                     [gate_up_fused] [gate_up_cublas] [qkv_cublas]
                                     [lm_head_argmax33|128] [lm_head_cublas33|128] [prefix_hash]

Each case captures 24 calls of one entry point into a CUDA graph, cycling over input sets
whose total exceeds the 126 MB L2 where the kernel is memory-bound, and prints the median
per-call time of five replays with the algorithmic bytes moved (one read of every input,
one write of every output). Shapes: 2080 tokens, hidden 2560, 32 query / 8 KV heads,
d = 128, inter 9728; attention cases are the config-3 halves (one 2048-token prefill row;
32 decode rows with contexts U[1024, 4096]) on 256-token pages.
"""

from __future__ import annotations

import math
import sys

import torch

from helios_b200 import _native, ops
from helios_b200.config import Qwen3Config
from helios_b200.paged_cache import KVPagePool, PackedBatchCache, PagedKVCache

T, H, HKV, D, HIDDEN, INTER = 2080, 32, 8, 128, 2560, 9728


def graph_time(calls, reps: int = 24, replays: int = 5) -> float:
    """Median microseconds per call over `replays` replays of a graph of `reps` calls."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for call in calls:
            call()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(reps):
            calls[i % len(calls)]()
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(replays):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end) * 1e3 / reps)
    return sorted(times)[len(times) // 2]


def _norm_rope(dev, g, T=T):
    cos, sin = torch.randn(40960, D, device=dev), torch.randn(40960, D, device=dev)
    qs, ks = torch.rand(D, device=dev) + 0.5, torch.rand(D, device=dev) + 0.5
    pages = 600

    def make():
        qkv = torch.randn(T, (H + 2 * HKV) * D, device=dev, generator=g).to(torch.bfloat16)
        q = qkv[:, :H * D].view(T, H, D)
        k = qkv[:, H * D:(H + HKV) * D].view(T, HKV, D)
        v = qkv[:, (H + HKV) * D:].view(T, HKV, D)
        kp = torch.zeros(pages, 256, HKV, D, dtype=torch.bfloat16, device=dev)
        vp = torch.zeros_like(kp)
        slots = torch.randperm(pages * 256, device=dev, generator=g)[:T].long()
        pos = torch.randint(0, 4096, (T,), device=dev, generator=g).long()
        qo = torch.empty(T, H, D, dtype=torch.bfloat16, device=dev)
        return lambda: ops.qk_norm_rope_append(q, k, v, q_scale=qs, k_scale=ks, eps=1e-6, cos=cos, sin=sin,
                                               positions=pos, write_slots=slots, q_out=qo, key_pool=kp,
                                               value_pool=vp)

    return [make() for _ in range(4)], T * (H + 2 * HKV) * D * 2 * 2


def _swiglu(dev, g, T=T):
    def make():
        gu = torch.randn(T, 2 * INTER, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty(T, INTER, dtype=torch.bfloat16, device=dev)
        return lambda: ops.swiglu(gu, out)

    return [make() for _ in range(4)], T * INTER * 3 * 2


def _add_rmsnorm(dev, g, T=T):
    scale = torch.rand(HIDDEN, device=dev) + 0.5

    def make():
        x = torch.randn(T, HIDDEN, device=dev, generator=g).to(torch.bfloat16)
        y = torch.randn_like(x)
        s, n = torch.empty_like(x), torch.empty_like(x)
        return lambda: ops.add_rmsnorm(x, y, scale, 1e-6, s, n)

    return [make() for _ in range(8)], T * HIDDEN * 2 * 4


def _gate_up(dev, g, fused: bool):
    """The MLP input side: gate|up projection + SwiGLU, fused (tcgen05) or cuBLAS + swiglu kernel."""
    import torch.nn.functional as F

    w = (torch.randn(2 * INTER, HIDDEN, device=dev, generator=g) / HIDDEN ** 0.5).to(torch.bfloat16)

    def make():
        x = torch.randn(T, HIDDEN, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty(T, INTER, dtype=torch.bfloat16, device=dev)
        if fused:
            return lambda: ops.gemm_swiglu(x, w, out)
        return lambda: ops.swiglu(F.linear(x, w), out)

    flops = 2 * T * HIDDEN * 2 * INTER
    return [make() for _ in range(2)], flops


def _qkv(dev, g):
    """The attention input side as the model runs it: the q|k|v projection on cuBLAS, then the
    per-head norm, RoPE and KV append kernel (b)."""
    import torch.nn.functional as F

    w = (torch.randn((H + 2 * HKV) * D, HIDDEN, device=dev, generator=g) / HIDDEN ** 0.5).to(torch.bfloat16)
    cos, sin = torch.randn(40960, D, device=dev), torch.randn(40960, D, device=dev)
    qs, ks = torch.rand(D, device=dev) + 0.5, torch.rand(D, device=dev) + 0.5
    pages = 600

    def make():
        x = torch.randn(T, HIDDEN, device=dev, generator=g).to(torch.bfloat16)
        kp = torch.zeros(pages, 256, HKV, D, dtype=torch.bfloat16, device=dev)
        vp = torch.zeros_like(kp)
        slots = torch.randperm(pages * 256, device=dev, generator=g)[:T].long()
        pos = torch.randint(0, 4096, (T,), device=dev, generator=g).long()
        qo = torch.empty(T, H, D, dtype=torch.bfloat16, device=dev)

        def call():
            qkv = F.linear(x, w)
            ops.qk_norm_rope_append(qkv[:, :H * D].view(T, H, D), qkv[:, H * D:(H + HKV) * D].view(T, HKV, D),
                                    qkv[:, (H + HKV) * D:].view(T, HKV, D), q_scale=qs, k_scale=ks, eps=1e-6,
                                    cos=cos, sin=sin, positions=pos, write_slots=slots, q_out=qo, key_pool=kp,
                                    value_pool=vp)
        return call

    flops = 2 * T * HIDDEN * (H + 2 * HKV) * D
    return [make() for _ in range(2)], flops


def _attention(dev, lengths, counts, sets):
    cfg = Qwen3Config(n_layers=1, context_length=8192)
    calls, kv_bytes = [], sum(l + c for l, c in zip(lengths, counts)) * HKV * D * 2 * 2
    for seed in range(sets):
        g = torch.Generator().manual_seed(seed)
        pages = sum(math.ceil((l + c) / 256) for l, c in zip(lengths, counts)) + 4
        pool = KVPagePool(cfg, pages, device=dev)
        pool.storage.normal_(0.0, 0.3)
        pool._free = list(reversed(torch.randperm(pages, generator=g).tolist()))  # pages in random order
        caches = []
        for length, count in zip(lengths, counts):
            cache = PagedKVCache(pool, length + count + 8)
            cache.pages.extend(pool.acquire(math.ceil(length / 256)))
            cache.length = length
            caches.append(cache)
        batch = PackedBatchCache(caches)
        batch.prepare_packed(counts)
        q = torch.randn(sum(counts), H, D, device=dev).to(torch.bfloat16)
        out = torch.empty_like(q)
        calls.append((lambda q=q, pool=pool, batch=batch, out=out, caches=caches:
                      ops.paged_attention(q, pool.keys[0], pool.values[0], batch, out)))
    return calls, kv_bytes


def _prefix_decode(dev, sets):
    """BASELINE config 4's decode attention: 128 rows share a 4096-token prefix (16 pages restored
    by page aliasing), each with its own tail of U[256, 1024] tokens, one query token per row.
    Reported bytes are the K/V the rows read (the shared pages once per row)."""
    cfg = Qwen3Config(n_layers=1, context_length=8192)
    rng = torch.Generator().manual_seed(3)
    tails = torch.randint(256, 1025, (128,), generator=rng).tolist()
    calls, kv_bytes = [], sum(4096 + t + 1 for t in tails) * HKV * D * 2 * 2
    for seed in range(sets):
        g = torch.Generator().manual_seed(seed)
        pages = 16 + sum(math.ceil((4096 + t + 1) / 256) - 16 for t in tails) + 4
        pool = KVPagePool(cfg, pages, device=dev)
        pool.storage.normal_(0.0, 0.3)
        pool._free = list(reversed(torch.randperm(pages, generator=g).tolist()))  # pages in random order
        prefix = PagedKVCache(pool, 4096)
        prefix.pages.extend(pool.acquire(16))
        prefix.length = 4096
        block = prefix.snapshot_block(0, 4096)
        caches = []
        for tail in tails:
            cache = PagedKVCache(pool, 4096 + tail + 8)
            cache.restore_blocks([block])  # the shared pages, aliased
            cache.pages.extend(pool.acquire(math.ceil((4096 + tail) / 256) - 16))
            cache.length = 4096 + tail
            caches.append(cache)
        batch = PackedBatchCache(caches)
        batch.prepare_packed([1] * len(caches))
        q = torch.randn(len(caches), H, D, device=dev).to(torch.bfloat16)
        out = torch.empty_like(q)
        calls.append((lambda q=q, pool=pool, batch=batch, out=out, caches=caches, prefix=prefix:
                      ops.paged_attention(q, pool.keys[0], pool.values[0], batch, out)))
    return calls, kv_bytes


def _sample(dev, g):
    """BASELINE config 4's sampling: 128 rows over the Qwen3 vocabulary (151936), temperature 0.2,
    top-p 0.95. Bytes: one read of the bf16 logits."""
    vocab, rows = 151936, 128

    def make():
        logits = (torch.randn(rows, vocab, device=dev, generator=g) * 3).to(torch.bfloat16)
        temperature = torch.full((rows,), 0.2, device=dev)
        top_p = torch.full((rows,), 0.95, device=dev)
        uniforms = torch.rand(rows, device=dev, generator=g)
        out = torch.empty(rows, dtype=torch.long, device=dev)
        return lambda: ops.sample(logits, temperature, top_p, uniforms, out)

    return [make() for _ in range(4)], rows * vocab * 2


def _lm_head(dev, g, rows: int, fused: bool):
    """The Qwen3-4B greedy head over `rows` logit rows: the tied [151936, 2560] lm_head and the
    argmax, either fused (hb_lm_head_argmax, no logits written) or cuBLAS + the sampler kernel at
    temperature 0. Bytes: one read of the weight."""
    vocab = 151936
    weight = (torch.randn(vocab, HIDDEN, device=dev, generator=g) * 0.02).to(torch.bfloat16)

    def make():
        x = torch.randn(rows, HIDDEN, device=dev, generator=g).to(torch.bfloat16)
        if fused:
            out = torch.empty(rows, dtype=torch.long, device=dev)
            return lambda: ops.lm_head_argmax(x, weight, out)
        zeros = torch.zeros(rows, device=dev)
        ones = torch.ones(rows, device=dev)
        out = torch.empty(rows, dtype=torch.long, device=dev)
        return lambda: ops.sample(torch.nn.functional.linear(x, weight), zeros, ones, zeros, out)

    return [make() for _ in range(2)], vocab * HIDDEN * 2


def _projection(dev, g, m: int, n: int, k: int):
    """One decode-tick projection [m, k] x [n, k]^T on cuBLAS, as the model runs it. Four
    weights cycled, 4 x n x k x 2 bytes, beyond L2 for the Qwen3-4B shapes."""
    def make():
        x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
        w = (torch.randn(n, k, device=dev, generator=g) / k ** 0.5).to(torch.bfloat16)
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        return lambda: torch.matmul(x, w.T, out=out)
    return [make() for _ in range(4)], n * k * 2


def _prefix_hash(dev, rows: int = 128):
    """BASELINE config 4's admission keys: 128 prompts of 4096 shared + U[256, 1024] own tokens,
    256-token blocks, keyed on the device (hb_hash_token_blocks). Bytes: the int32 tokens read."""
    from helios_b200 import prefix_index

    rng = torch.Generator().manual_seed(3)
    shared = torch.randint(0, 151936, (4096,), generator=rng).tolist()
    prompts = [shared + torch.randint(0, 151936, (int(n),), generator=rng).tolist()
               for n in torch.randint(256, 1025, (rows,), generator=rng)]
    tokens, offsets, block_offsets, _ = prefix_index._flatten(prompts, 256)
    d_tok = torch.from_numpy(tokens).to(dev)
    d_off = torch.from_numpy(offsets).to(dev)
    d_boff = torch.from_numpy(block_offsets).to(dev)
    digests = torch.empty((int(block_offsets[-1]), 32), dtype=torch.uint8, device=dev)

    def call():
        rc = _native.load().hb_hash_token_blocks(d_tok.data_ptr(), d_off.data_ptr(), rows, 256, d_boff.data_ptr(),
                                                 digests.data_ptr(), torch.cuda.current_stream().cuda_stream)
        _native.check(rc, "hb_hash_token_blocks")

    return [call], tokens.size * 4


def main(argv: list[str]) -> None:
    if not torch.cuda.is_available():
        raise SystemExit("the microbenchmarks need a CUDA device")
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    rng = torch.Generator().manual_seed(3)
    decode_lengths = torch.randint(1024, 4097, (32,), generator=rng).tolist()
    cases = {
        "norm_rope": lambda: _norm_rope(dev, g),
        "swiglu": lambda: _swiglu(dev, g),
        "add_rmsnorm": lambda: _add_rmsnorm(dev, g),
        # the same row kernels at a decode tick's 128 rows: latency-bound
        "norm_rope128": lambda: _norm_rope(dev, g, 128),
        "swiglu128": lambda: _swiglu(dev, g, 128),
        "add_rmsnorm128": lambda: _add_rmsnorm(dev, g, 128),
        "prefill": lambda: _attention(dev, [0], [2048], 1),
        **{f"proj_{name}{m}": (lambda m=m, n=n, k=k: _projection(dev, g, m, n, k))
           for name, n, k in (("qkv", 6144, 2560), ("o", 2560, 4096), ("gateup", 19456, 2560), ("down", 2560, 9728))
           for m in (32, 128, 256)},
        "decode": lambda: _attention(dev, decode_lengths, [1] * 32, 2),
        "mixed": lambda: _attention(dev, decode_lengths + [0], [1] * 32 + [2048], 2),
        "prefix_decode": lambda: _prefix_decode(dev, 2),
        "sample": lambda: _sample(dev, g),
        "gate_up_fused": lambda: _gate_up(dev, g, True),
        "gate_up_cublas": lambda: _gate_up(dev, g, False),
        "qkv_cublas": lambda: _qkv(dev, g),
        "prefix_hash": lambda: _prefix_hash(dev),
        "lm_head_argmax33": lambda: _lm_head(dev, g, 33, True),
        "lm_head_cublas33": lambda: _lm_head(dev, g, 33, False),
        "lm_head_argmax128": lambda: _lm_head(dev, g, 128, True),
        "lm_head_cublas128": lambda: _lm_head(dev, g, 128, False),
    }
    for arg in argv or list(cases):
        # "mixed:48" times a case with the decode grid keeping 48 SMs beside the prefill grid
        # (hb_attention_set_overlap; 0 runs them one after the other).
        name, _, overlap = arg.partition(":")
        if overlap:
            _native.check(_native.load().hb_attention_set_overlap(int(overlap)), "hb_attention_set_overlap")
            name_shown = arg
        else:
            name_shown = name
        calls, nbytes = cases[name]()
        with torch.inference_mode():
            us = graph_time(calls)
        if name.startswith(("gate_up", "qkv")):  # compute-bound: report TFLOP/s
            print(f"{name_shown:14s} {us:8.2f} us/call   {nbytes / us / 1e6:8.1f} TFLOP/s", flush=True)
        else:
            print(f"{name_shown:12s} {us:8.2f} us/call   {nbytes / 1e6:8.1f} MB   {nbytes / us / 1e3:8.1f} GB/s",
                  flush=True)
        del calls
        torch.cuda.empty_cache()
    status = _native.device_status()
    if status:
        raise SystemExit(f"device status: {_native.describe_status(status)}")


if __name__ == "__main__":
    main(sys.argv[1:])
