"""Benchmark of the B200 packed mixed-batch tick (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload: Qwen3-4B architecture, random-init bf16 weights;
one tick = 32 decode rows (contexts uniform in [1024, 4096], their K/V already
in the paged pool) + one 2048-token prefill chunk at offset 0 = 2080 tokens.
A step is one tick: tick packing, 36 layers and the greedy ids of the 33 trailing
rows (lm_head GEMM with the argmax in its epilogue). Each tick starts a fresh prefill request (its pages are
recycled afterwards) and advances every decode row by one token. The host half
of each tick (page acquisition, descriptor upload, tick packing) runs every
step; the device half replays from a CUDA graph captured during warm-up
(helios_b200.graphs), with the tick's work counts read on the device.

  value   tokens/s with the step's token ids already on the device, timed with
          CUDA events over K steps (max over ranks), summed over replicas.
  e2e     the same ticks through the public API (``Decoder.packed_caches_greedy`` with
          host token lists, device->host read of the sampled ids).
  roofline  the split-K decode attention kernel at BASELINE config 2 (64 rows,
          contexts U[512, 8192], 32/8 heads, d=128, 4096-page pool), HBM-bound:
          algorithmic bytes / CUDA-event time against the measured copy peak.
  cpu_baseline  the same tick on the reference's own packed CPU path, imported
          unchanged from baseline/_ref (else the oracle's CPU restatement), timed on a
          bounded sample of decoder layers and scaled to 36 (rank 0, N=1 only).
  per_rank  each replica's own ms per tick and median SM clock (N>1: what limits scaling).
  config4  BASELINE config 4 end to end (helios_b200.workloads.config4): restore cost of
          128 prefix-hit requests, their tail prefill, 128 sampled decode steps.
  config5  BASELINE config 5 at 64 req/s per GPU, 256 requests per GPU, on the reference's
          Engine over this path, all replicas (helios_b200.load): tokens/s and p50 TTFT.
  reference_gpu_dense  the reference's own GPU path for the same tick (its dense-KV CUDA
          path, imported unchanged; its paged varlen_attn path needs torch >= 2.13).

Multi-GPU: one process per GPU (torchrun), independent replicas, no collective
on the data path; the process group only aligns the ranks and takes max time.
``--impl reference`` times the reference's own packed CPU path (imported unchanged; the
oracle's restatement when the reference is absent) on the host cores, rank 0 only (other
ranks exit), and prints the same metric with ``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "packed-tick tokens/s (Qwen3-4B shape, 32 decode rows + 2048-token prefill chunk)"
UNIT = "tokens/s"
DECODE_ROWS = 32
PREFILL = 2048
CONTEXT = (1024, 4096)
TOKENS_PER_STEP = DECODE_ROWS + PREFILL
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
DATA = "synthetic: random-init weights, uniform token ids, random K/V standing in for the decode rows' prefill"
CONFIG5_RATE = 64.0            # requests/s per GPU for the bench's config-5 point
CONFIG5_REQUESTS_PER_GPU = 256


_T0 = time.time()


def stage(text: str) -> None:
    """Progress line on stderr, tagged with the rank and seconds since start (rank 0's
    JSON line stays the only stdout output)."""
    print(f"[bench rank {os.environ.get('RANK', '0')} +{time.time() - _T0:6.1f}s] {text}", file=sys.stderr, flush=True)


def peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


# ------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms; the summary keeps the
    samples taken between mark_start() and mark_end() (the timed region)."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu_index = gpu_index
        self.proc = None
        self.file = None
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        deadline = time.time() + 5.0  # wait for the first sample so the region is covered
        while time.time() < deadline and self.proc.poll() is None and not Path(self.file.name).read_text():
            time.sleep(0.02)
        return self

    def mark_start(self) -> None:
        self.t0 = time.time()

    def mark_end(self) -> None:
        self.t1 = time.time()
        time.sleep(0.06)  # let the sample after the region land

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary_cached(self) -> dict:
        if not hasattr(self, "_summary"):
            self._summary = self.summary()
        return self._summary

    def summary(self) -> dict:
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10 and parts[1] == str(self.gpu_index):
                rows.append(parts)
        os.unlink(self.file.name)

        def stamp(text):
            try:
                return datetime.datetime.strptime(text, "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                return None

        if self.t0 is not None and self.t1 is not None:
            inside = [r for r in rows if (t := stamp(r[0])) is not None and self.t0 - 0.05 <= t <= self.t1 + 0.05]
            rows = inside or rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[6 + i].lower() in ("active", "1")})

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [v for v in (num(r[2]) for r in rows) if v is not None]
        mx = [v for v in (num(r[3]) for r in rows) if v is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------- B200 arm
def build_replica(device: torch.device, seed: int, steps_total: int):
    from helios_b200.config import qwen3_4b_config
    from helios_b200.decode import Decoder
    from helios_b200.model import Qwen3Model
    from helios_b200.paged_cache import KVPagePool, PagedKVCache

    cfg = qwen3_4b_config()
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen3Model(cfg).eval()
    # The device half of each tick replays from a CUDA graph (helios_b200.graphs); the
    # host half (page acquisition, descriptor upload, tick packing) runs every tick.
    model.enable_cuda_graphs()
    g = torch.Generator().manual_seed(seed)
    contexts = torch.randint(CONTEXT[0], CONTEXT[1] + 1, (DECODE_ROWS,), generator=g).tolist()
    pages = sum(math.ceil((c + steps_total + 1) / 256) for c in contexts) + math.ceil(PREFILL / 256) + 8
    pool = KVPagePool(cfg, pages, device=device)
    # The decode rows' context K/V: finite random values in every page (stands in for their prefill).
    gen = torch.Generator(device=device).manual_seed(seed)
    for layer in range(cfg.n_layers):
        pool.storage[layer].normal_(0.0, 0.3, generator=gen)
    decoder = Decoder(model)
    decoder.page_pool = pool
    caches = []
    for ctx in contexts:
        cache = PagedKVCache(pool, ctx + steps_total + 1)
        cache.pages.extend(pool.acquire(math.ceil((ctx - 1) / 256)))
        cache.length = ctx - 1
        caches.append(cache)
    pending = torch.randint(0, cfg.vocab_size, (DECODE_ROWS,), generator=g).tolist()
    chunk = torch.randint(0, cfg.vocab_size, (PREFILL,), generator=g).tolist()
    return model, decoder, pool, caches, pending, chunk


class TickRunner:
    """Runs ticks either through the public API (host lists) or with device-resident ids."""

    def __init__(self, device, model, decoder, pool, caches, pending, chunk):
        from helios_b200.paged_cache import PackedBatchCache

        self.device, self.model, self.decoder, self.pool = device, model, decoder, pool
        self.caches, self.pending, self.chunk = caches, pending, chunk
        self.batch = PackedBatchCache(caches)
        self.chunk_dev = torch.tensor(chunk, dtype=torch.long, device=device)
        self.pending_dev = torch.tensor(pending, dtype=torch.long, device=device)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.launches = 0

    def _fresh_prefill(self):
        from helios_b200.paged_cache import PagedKVCache

        return PagedKVCache(self.pool, PREFILL + 64)

    def device_step(self):
        """Token ids stay on the device; metadata still goes through tick packing."""
        prefill = self._fresh_prefill()
        batch = self.batch
        batch.caches, batch.batch_size = tuple(self.caches) + (prefill,), DECODE_ROWS + 1
        with torch.inference_mode():
            ids = torch.cat([self.pending_dev, self.chunk_dev]).unsqueeze(0)
            batch.prepare_packed([1] * DECODE_ROWS + [PREFILL])
            sampled = self.model.greedy_ids(ids, batch)
            self.pending_dev = sampled[:DECODE_ROWS]
        self.launches = self._count_launches(batch)
        batch.caches = ()
        prefill.close()

    def api_step(self):
        """Public API with host buffers: token lists in, sampled ids back on the host."""
        prefill = self._fresh_prefill()
        chunks = [[t] for t in self.pending] + [self.chunk]
        with torch.inference_mode():
            ids = self.decoder.packed_caches_greedy(self.caches + [prefill], chunks).cpu().tolist()
        self.pending = ids[:DECODE_ROWS]
        batch = self.decoder._packed_batch
        # token ids + tick descriptor (rows and new arena entries)
        self.h2d_bytes = 8 * TOKENS_PER_STEP + batch.uploaded_bytes
        self.d2h_bytes = 8 * (DECODE_ROWS + 1)
        self.launches = self._count_launches(batch)
        prefill.close()

    def _count_launches(self, batch) -> int:
        attention = (batch.num_decode_items > 0) + (batch.num_decode_items > 0 and batch.partial_records > 0) \
            + (batch.num_prefill_items > 0) + (batch.num_prefix_items > 0)
        per_layer = 1 + attention + 2 + 1  # norm/rope/append, attention, add_rmsnorm x2, swiglu
        # tick pack, embed, first norm, the layers, the lm_head GEMM with the argmax and its finalize
        return 3 + per_layer * self.model.config.n_layers + 2


def time_steps(step, steps: int, device: torch.device, *, all_ranks: bool = True) -> float:
    """Seconds for ``steps`` calls of ``step``, CUDA events on the current stream. With
    ``all_ranks`` every rank must call it (the region is bracketed by barriers); legs that
    rank 0 runs alone pass False, so they take no collective step."""
    from helios_b200 import replicas

    torch.cuda.synchronize(device)
    if all_ranks:
        replicas.barrier(device)
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        torch.cuda.nvtx.range_push("tick")  # lets a profiler select exactly the timed ticks
        step()
        torch.cuda.nvtx.range_pop()
    end.record()
    torch.cuda.synchronize(device)
    if all_ranks:
        replicas.barrier(device)
    torch.cuda.synchronize(device)
    return start.elapsed_time(end) / 1000.0


def graph_seconds_per_call(call, device: torch.device, iters: int, warmup: int = 3) -> float:
    """Device time of one ``call`` (a launch sequence of one kernel call) with no host gaps:
    ``iters`` calls captured in one CUDA graph, replayed five times between CUDA events on
    the capturing stream; the median replay is divided by ``iters``. Eager back-to-back calls
    would also time the host's launch work between short kernels."""
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(warmup):
            call()
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(iters):
            call()
    graph.replay()
    torch.cuda.synchronize(device)
    times = []
    stream = torch.cuda.current_stream(device)
    for _ in range(5):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        graph.replay()
        end.record(stream)
        torch.cuda.synchronize(device)
        times.append(start.elapsed_time(end) / 1e3 / iters)
    del graph
    return sorted(times)[2]


def measured_traffic(kernel: str) -> int | None:
    """DRAM bytes (read + write) per launch of `kernel` from the committed ncu capture of the
    same workload (profiles/roofline_traffic.json), or None when there is none."""
    path = ROOT / "profiles" / "roofline_traffic.json"
    try:
        entry = json.loads(path.read_text())[kernel]
        return int(entry["dram_bytes_read_per_launch"]) + int(entry["dram_bytes_write_per_launch"])
    except (OSError, KeyError, ValueError):
        return None


def prefill_attention_roofline(device: torch.device, peak_tflops: float, iters: int = 20) -> dict:
    """The prefill half of BASELINE config 3 through the C ABI: one 2048-token row at offset 0,
    32/8 heads, d=128 (tensor-bound). Algorithmic FLOPs per call: 4 * H * d * causal keys."""
    from helios_b200 import ops
    from helios_b200.config import Qwen3Config
    from helios_b200.paged_cache import KVPagePool, PackedBatchCache, PagedKVCache

    cfg = Qwen3Config(n_layers=1, context_length=PREFILL + 64)
    pool = KVPagePool(cfg, math.ceil(PREFILL / 256) + 1, device=device)
    gen = torch.Generator(device=device).manual_seed(2)
    pool.storage.normal_(0.0, 0.3, generator=gen)
    batch = PackedBatchCache([PagedKVCache(pool, PREFILL)])
    with torch.inference_mode():
        batch.prepare_packed([PREFILL])
        q = torch.randn(PREFILL, cfg.n_heads, cfg.head_dim, device=device, generator=gen).to(torch.bfloat16)
        out = torch.empty_like(q)
        seconds = graph_seconds_per_call(lambda: ops.paged_attention(q, pool.keys[0], pool.values[0], batch, out),
                                         device, iters)
    flops = 4 * cfg.n_heads * cfg.head_dim * (PREFILL * (PREFILL + 1) // 2)
    achieved = flops / seconds / 1e12
    del pool, batch
    torch.cuda.empty_cache()
    return {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak_tflops, "unit": "TFLOP/s",
            "frac": round(achieved / peak_tflops, 4), "kernel": "prefill_attention_kernel (tcgen05/TMEM)",
            "workload": "BASELINE config 3 prefill half: one 2048-token row at offset 0, 32/8 heads, d=128",
            "flops_per_call": flops, "us_per_call": round(seconds * 1e6, 2),
            "timing": f"median of 5 CUDA-graph replays of {iters} calls, CUDA events"}


def decode_attention_roofline(device: torch.device, peak_gbs: float, iters: int = 20) -> dict:
    """BASELINE config 2 through the C ABI: 64 rows x 1 query, contexts U[512, 8192], 4096 pages."""
    from helios_b200 import ops
    from helios_b200.workloads import config2_batch

    pool, batch, q, contexts = config2_batch(device)
    with torch.inference_mode():
        out = torch.empty_like(q)
        seconds = graph_seconds_per_call(lambda: ops.paged_attention(q, pool.keys[0], pool.values[0], batch, out),
                                         device, iters)
    kv_bytes = sum(contexts) * 8 * 128 * 2 * 2
    io_bytes = 2 * 64 * 32 * 128 * 2 + 64 * batch.block_table.shape[1] * 4
    achieved = (kv_bytes + io_bytes) / seconds / 1e9
    info = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
            "frac": round(achieved / peak_gbs, 4), "traffic": measured_traffic("decode_attention_kernel"),
            "kernel": "decode_attention_kernel (+ decode_combine_kernel), hb_paged_attention on decode rows",
            "workload": "BASELINE config 2: 64 rows x 1 query, context U[512,8192], 32/8 heads, d=128, 4096 pages",
            "algorithmic_bytes_per_call": kv_bytes + io_bytes, "us_per_call": round(seconds * 1e6, 2),
            "split_keys": batch.split_keys, "decode_items": batch.num_decode_items,
            "timing": f"median of 5 CUDA-graph replays of {iters} calls, CUDA events"}
    del pool, batch
    torch.cuda.empty_cache()
    return info


# ------------------------------------------------------------------------- the reference's own code
def reference_package():
    """``helios_b200.reference_engine`` with the reference importable (baseline/_ref or
    HELIOS_REFERENCE_SRC), else None."""
    try:
        from helios_b200 import reference_engine

        reference_engine.import_reference()
        return reference_engine
    except Exception:  # noqa: BLE001 - any import failure means the reference is absent
        return None


def _tile_fill(t: torch.Tensor, gen: torch.Generator, scale: float) -> None:
    """Fill ``t`` with a tiled block of N(0, scale) values (finite, no denormals): timing
    inputs only, far cheaper than the reference's serial initialisation on the CPU."""
    block = (torch.randn(1 << 16, generator=gen) * scale).to(t.dtype)
    flat = t.view(-1)
    reps = -(-flat.numel() // block.numel())
    flat.copy_(block.repeat(reps)[:flat.numel()])


class ReferenceCpuTick:
    """BASELINE config 3's tick on the reference's own packed CPU path, imported unchanged
    (``Decoder.packed_caches`` -> ``PackedBatchCache.prepare_packed`` -> ``Qwen3Model._forward_packed``
    with the CPU branch of ``PackedBatchCache.attend``, src/helios/runtime/qwen3/decode.py:260-291,
    paged_cache.py:418-546), on ``layers`` decoder layers of the Qwen3-4B shape. Forward hooks
    time each decoder layer, so a step's time scales to 36 layers as
    (whole step - its layers) + 36 x (mean layer time)."""

    def __init__(self, layers: int, seed: int = 0, threads: int | None = None, steps: int = 64) -> None:
        if reference_package() is None:
            raise RuntimeError("the reference package is not importable")
        from helios.runtime.qwen3.config import Qwen3Config as RefConfig
        from helios.runtime.qwen3.decode import Decoder as RefDecoder
        from helios.runtime.qwen3.layers import rope_parameters as ref_rope
        from helios.runtime.qwen3.model import Qwen3Model as RefModel
        from helios.runtime.qwen3.paged_cache import KVPagePool as RefPool
        from helios.runtime.qwen3.paged_cache import PagedKVCache as RefCache

        self.threads = threads or os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.layers = layers
        cfg = RefConfig(n_layers=layers)
        with torch.device("meta"):
            model = RefModel(cfg)
        model = model.to_empty(device="cpu")
        model.output.weight = model.token_embedding.weight
        gen = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, param in model.named_parameters():
                if name.endswith("scale"):
                    param.fill_(1.0)
                else:
                    _tile_fill(param, gen, 0.02 if "embedding" not in name else 1.0)
            cos, sin = ref_rope(cfg)
            model.cos.copy_(cos)
            model.sin.copy_(sin)
        self.model = model.eval()
        g = torch.Generator().manual_seed(seed)
        contexts = torch.randint(CONTEXT[0], CONTEXT[1] + 1, (DECODE_ROWS,), generator=g).tolist()
        pages = sum(math.ceil((c + steps + 1) / 256) for c in contexts) + math.ceil((PREFILL + 8) / 256) + 2
        self.pool = RefPool(cfg, pages, device=torch.device("cpu"))
        for layer in range(layers):
            _tile_fill(self.pool.keys[layer], gen, 0.3)
            _tile_fill(self.pool.values[layer], gen, 0.3)
        self.caches = []
        for ctx in contexts:
            cache = RefCache(self.pool, ctx + steps + 1)
            cache.pages.extend(self.pool.acquire(math.ceil((ctx - 1) / 256)))
            cache.length = ctx - 1
            self.caches.append(cache)
        self.decoder = RefDecoder(self.model)
        self.decoder.page_pool = self.pool
        self.cache_cls = RefCache
        self.pending = torch.randint(0, cfg.vocab_size, (DECODE_ROWS,), generator=g).tolist()
        self.chunk = torch.randint(0, cfg.vocab_size, (PREFILL,), generator=g).tolist()
        self._block_seconds = 0.0
        self._started = 0.0

        def pre(module, args):
            self._started = time.perf_counter()

        def post(module, args, output):
            self._block_seconds += time.perf_counter() - self._started

        for block in self.model.blocks:
            block.register_forward_pre_hook(pre)
            block.register_forward_hook(post)

    def step(self) -> float:
        """One tick; returns its time scaled to 36 decoder layers."""
        prefill = self.cache_cls(self.pool, PREFILL + 8)
        self._block_seconds = 0.0
        started = time.perf_counter()
        logits = self.decoder.packed_caches(self.caches + [prefill], [[t] for t in self.pending] + [self.chunk])
        ids = logits.float().argmax(-1).tolist()
        total = time.perf_counter() - started
        prefill.close()
        self.pending = ids[:DECODE_ROWS]
        layer = self._block_seconds / self.layers
        return total - self._block_seconds + 36 * layer


def reference_gpu_dense(device: torch.device, steps: int, warmup: int = 3, seed: int = 0) -> dict:
    """The reference's own GPU path for BASELINE config 3's tick, imported unchanged: its
    paged ``varlen_attn`` path needs torch >= 2.13 (``block_table``), absent from this image,
    so the comparator is its dense-KV CUDA path (what its decoder runs without a page pool):
    ``Decoder.decode_caches`` over 32 dense caches (``_decode_dense``: one batched decode
    forward, src/helios/runtime/qwen3/decode.py:293-320) plus one 2048-token prefill through
    ``Decoder._forward_cache`` (SDPA, layers.py:169-191), greedy ids read back each step,
    eager as the reference runs. Random-init Qwen3-4B weights; random K/V in the decode rows'
    contexts. CUDA events around ``steps`` ticks."""
    if reference_package() is None:
        raise RuntimeError("the reference package is not importable")
    from helios.runtime.qwen3.cache import KVCache
    from helios.runtime.qwen3.config import Qwen3Config as RefConfig
    from helios.runtime.qwen3.decode import Decoder as RefDecoder
    from helios.runtime.qwen3.model import Qwen3Model as RefModel

    cfg = RefConfig()
    torch.manual_seed(seed)
    with torch.device(device):
        model = RefModel(cfg).eval()
    decoder = RefDecoder(model)
    g = torch.Generator().manual_seed(seed)
    contexts = torch.randint(CONTEXT[0], CONTEXT[1] + 1, (DECODE_ROWS,), generator=g).tolist()
    total = warmup + steps + 1
    gen = torch.Generator(device=device).manual_seed(seed)
    caches = []
    for ctx in contexts:
        cache = KVCache(cfg, ctx + total, device=device)
        for layer in cache._layers:
            layer.keys[:, :, :ctx - 1].normal_(0.0, 0.3, generator=gen)
            layer.values[:, :, :ctx - 1].normal_(0.0, 0.3, generator=gen)
        cache.length = ctx - 1
        caches.append(cache)
    pending = torch.randint(0, cfg.vocab_size, (DECODE_ROWS,), generator=g).tolist()
    chunk = torch.randint(0, cfg.vocab_size, (1, PREFILL), generator=g).to(device)

    def tick():
        nonlocal pending
        with torch.inference_mode():
            decode_logits = decoder.decode_caches(caches, pending)
            prefill_logits = decoder._forward_cache(chunk, KVCache(cfg, PREFILL + 8, device=device))[:, -1, :]
            ids = torch.cat([decode_logits.argmax(-1), prefill_logits.argmax(-1)]).tolist()
        pending = ids[:DECODE_ROWS]

    for _ in range(warmup):
        tick()
    seconds = time_steps(tick, steps, device, all_ranks=False)  # rank 0 alone runs this leg
    del caches, model, decoder
    torch.cuda.empty_cache()
    return {"value": round(TOKENS_PER_STEP * steps / seconds, 1), "unit": UNIT,
            "ms_per_step": round(1e3 * seconds / steps, 3), "steps": steps,
            "path": "the reference's dense-KV CUDA path imported unchanged (Decoder.decode_caches -> _decode_dense "
                    "for the 32 decode rows + Decoder._forward_cache SDPA prefill of the 2048-token chunk), eager; "
                    "its varlen_attn paged path needs torch >= 2.13 and is not in this image"}


# ------------------------------------------------------------------------- CPU (oracle) tick
def cpu_tick_sample(layers: int, seed: int = 0, threads: int | None = None) -> dict:
    """The oracle's dense CPU restatement of the same tick on ``layers`` decoder layers.

    Returns the seconds per sampled layer and of the rest of the tick (embedding,
    final norm, logits of the 33 trailing rows), so the 36-layer tick can be scaled.
    """
    from oracle.metadata import pack_tick
    from oracle.model import OracleConfig, OracleModel, build_state_dict
    from oracle.numerics import rms_norm

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = OracleConfig()
    sd = build_state_dict(cfg, seed, layers=layers)
    model = OracleModel(cfg, sd, layers=layers)
    g = torch.Generator().manual_seed(seed)
    contexts = torch.randint(CONTEXT[0], CONTEXT[1] + 1, (DECODE_ROWS,), generator=g).tolist()
    lengths = [c - 1 for c in contexts] + [0]
    counts = [1] * DECODE_ROWS + [PREFILL]
    tables, at = [], 0
    for length, count in zip(lengths, counts):
        n = math.ceil((length + count) / 256)
        tables.append(list(range(at, at + n)))
        at += n
    meta = pack_tick(lengths, counts, tables, [l + c + 8 for l, c in zip(lengths, counts)])
    kp = [(torch.randn(at, 256, 8, 128, generator=g) * 0.3).to(torch.bfloat16) for _ in range(layers)]
    vp = [(torch.randn(at, 256, 8, 128, generator=g) * 0.3).to(torch.bfloat16) for _ in range(layers)]
    ids = torch.randint(0, cfg.vocab_size, (TOKENS_PER_STEP,), generator=g)
    with torch.inference_mode():
        t0 = time.perf_counter()
        x = sd["token_embedding.weight"][ids]
        t1 = time.perf_counter()
        for i in range(layers):
            x = model._block(i, x, kp[i], vp[i], meta)
        t2 = time.perf_counter()
        rows = x[torch.as_tensor(meta["logit_indices"])]
        logits = torch.nn.functional.linear(rms_norm(rows, sd["final_norm.scale"], cfg.rms_norm_eps),
                                            sd["output.weight"])
        logits.float().argmax(-1)
        t3 = time.perf_counter()
    return {"layer_seconds": (t2 - t1) / layers, "rest_seconds": (t1 - t0) + (t3 - t2), "threads": threads,
            "layers": layers}


def cpu_tokens_per_s(sample: dict, layers_total: int = 36) -> float:
    return TOKENS_PER_STEP / (sample["layer_seconds"] * layers_total + sample["rest_seconds"])


def cpu_baseline() -> dict:
    if reference_package() is not None:
        first = ReferenceCpuTick(1)
        first.step()
        one = first.step()
        layer_s = first._block_seconds
        # Grow the sample toward ~10 s of CPU work, capped at 4 layers.
        layers = int(max(1, min(4, 10.0 // max(layer_s, 1e-3))))
        tick = ReferenceCpuTick(layers) if layers > 1 else first
        if layers > 1:
            tick.step()
        seconds = statistics.mean(tick.step() for _ in range(2)) if layers > 1 else one
        return {"value": round(TOKENS_PER_STEP / seconds, 2), "unit": UNIT, "cores": tick.threads,
                "kind": "reference",
                "sample": f"the reference's own packed CPU path imported unchanged (bf16), {layers} of 36 decoder "
                          f"layers of the full 2080-token tick timed by forward hooks and scaled to 36 layers"}
    first = cpu_tick_sample(1)
    # Grow the sample toward ~10 s of CPU work, capped at 4 layers.
    layers = int(max(1, min(4, 10.0 // max(first["layer_seconds"], 1e-3))))
    sample = cpu_tick_sample(layers) if layers > 1 else first
    value = cpu_tokens_per_s(sample)
    return {"value": round(value, 2), "unit": UNIT, "cores": sample["threads"], "kind": "port",
            "sample": f"{sample['layers']} of 36 decoder layers of the full 2080-token tick (+ embedding and "
                      f"33 logit rows), scaled to 36 layers; oracle dense restatement, bf16 on CPU"}


def workload_config(n: int) -> dict:
    return {"workload": "BASELINE config 3: full mixed packed tick", "model": "Qwen3-4B architecture, random init",
            "global_batch": (DECODE_ROWS + 1) * n, "seq_len": PREFILL, "decode_rows": DECODE_ROWS,
            "decode_context": f"U[{CONTEXT[0]},{CONTEXT[1]}]", "prefill_chunk": PREFILL,
            "tokens_per_step": TOKENS_PER_STEP, "parallelism": f"replicas x{n} (no data-path collective)",
            "l2": "inputs larger than L2: each step streams ~8 GB of weights and ~12 GB of KV",
            "cuda_graphs": "device half of each tick replayed from a CUDA graph; host half and tick packing eager"}


def run_reference(args) -> None:
    from helios_b200 import replicas

    rank, _, _ = replicas.world()
    if rank != 0:
        return
    times = []
    if reference_package() is not None:
        tick = ReferenceCpuTick(1, steps=args.warmup + args.steps + 1)
        for _ in range(args.warmup):
            tick.step()
        times = [tick.step() for _ in range(args.steps)]
        kind, cores = "reference", tick.threads
        sample_text = ("each step: the full 2080-token tick through the reference's own packed CPU path "
                       "(imported unchanged, bf16) with 1 of 36 decoder layers, scaled to 36 layers by its "
                       "measured layer time")
    else:
        for _ in range(args.warmup):
            cpu_tick_sample(1)
        sample = None
        for _ in range(args.steps):
            sample = cpu_tick_sample(1)
            times.append(TOKENS_PER_STEP / cpu_tokens_per_s(sample))
        kind, cores = "port", sample["threads"]
        sample_text = ("each step: 1 of 36 decoder layers of the full tick (+ embedding and logit rows), scaled to "
                       "36 layers; the oracle's CPU restatement of the reference algorithm (reference not importable)")
    value = TOKENS_PER_STEP / statistics.mean(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * statistics.mean(times), 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": DATA,
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": sample_text},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args) -> None:
    from helios_b200 import replicas

    rank, size, local = replicas.world()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if size > 1:  # N replicas share the host's cores (their engines' host work in config 5)
        torch.set_num_threads(max(1, (os.cpu_count() or 1) // size))
    # Rank 0 alone runs the rooflines and configs 4 and the reference's GPU path while the
    # others wait at a barrier, so the group's timeout leaves room for those stages.
    replicas.init("nccl" if size > 1 else "gloo", timeout_s=600.0)
    pk, pk_kind = peaks()
    # The two attention kernels timed alone (against the burst peaks), before the long tick loop
    # holds the GPU at its power cap; rank 0 only, the others wait at the barrier.
    roof = prefill_roof = None
    if rank == 0:
        stage("rooflines")
        roof = decode_attention_roofline(device, pk["hbm_gbs"])
        prefill_roof = prefill_attention_roofline(device, pk["bf16_tflops"])
        roof["peak_kind"] = prefill_roof["peak_kind"] = pk_kind
    replicas.barrier(device)
    stage("replica build")
    steps_total = args.warmup * 2 + args.steps * 2 + 4
    model, decoder, pool, caches, pending, chunk = build_replica(device, seed=1000 + rank, steps_total=steps_total)
    runner = TickRunner(device, model, decoder, pool, caches, pending, chunk)
    with ClockSampler(local) as clocks:
        stage("warm-up ticks")
        for _ in range(args.warmup):
            runner.device_step()
        torch.cuda.synchronize(device)
        clocks.mark_start()
        seconds = time_steps(runner.device_step, args.steps, device)
        clocks.mark_end()
    seconds_local = seconds
    seconds = replicas.max_over_ranks(seconds, device)
    value = size * TOKENS_PER_STEP * args.steps / seconds
    stage(f"timed ticks done: {1e3 * seconds_local / args.steps:.3f} ms per tick")
    # End to end through the public API, host token lists in, sampled ids out.
    for _ in range(max(3, args.warmup // 2)):  # eager tick, graph capture, first replay
        runner.api_step()
    e2e_seconds = replicas.max_over_ranks(time_steps(runner.api_step, args.steps, device), device)
    e2e_value = size * TOKENS_PER_STEP * args.steps / e2e_seconds
    h2d, d2h, launches = runner.h2d_bytes, runner.d2h_bytes, runner.launches
    own_ms = 1e3 * seconds_local / args.steps
    flops = 2 * 3.633e9 * TOKENS_PER_STEP  # dense projections + MLP, all layers
    del runner, model, decoder, pool, caches
    torch.cuda.empty_cache()
    per_rank = replicas.gather_objects({"rank": rank, "ms_per_step": round(own_ms, 3),
                                        "sm_mhz": clocks.summary_cached().get("sm_mhz")}, device)
    extras = {}
    if not args.no_extras:
        extras = run_extras(args, device, rank, size)
    if rank == 0 and size == 1 and not args.no_cpu:
        stage("CPU baseline")
    cpu = cpu_baseline() if (rank == 0 and size == 1 and not args.no_cpu) else None
    if rank == 0:
        step_s = seconds / args.steps
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": size, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1000 * step_s, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": DATA,
            "config": workload_config(size),
            "roofline": roof,
            "prefill_roofline": prefill_roof,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(1000 * e2e_seconds / args.steps, 3)},
            "gpu_launches": args.steps * launches,
            "clocks": clocks.summary_cached(),
            "per_rank": per_rank,
            "tick_tensor_roofline": {"bound": "tensor", "flops_per_step": flops,
                                     "achieved_tflops": round(flops / step_s / 1e12, 1),
                                     "peak_tflops": pk["bf16_tflops_sustained"], "peak_kind": pk_kind,
                                     "frac": round(flops / step_s / 1e12 / pk["bf16_tflops_sustained"], 4)},
            **extras,
        }
        print(json.dumps(line), flush=True)
    replicas.shutdown()


def run_extras(args, device: torch.device, rank: int, size: int) -> dict:
    """The other BASELINE configs and the reference's own GPU path, each under its own key.
    Every rank takes the same collective steps (config 5 runs on all replicas)."""
    out = {}
    from helios_b200 import replicas

    # Config 4 and the reference's GPU path do not depend on N: one GPU measures them (N=1).
    if rank == 0 and size == 1:
        from helios_b200.workloads import config4

        try:
            stage("config 4")
            out["config4"] = config4(steps=128, device=device)
        except Exception as error:  # noqa: BLE001 - reported in the line, the headline stands
            out["config4"] = {"error": f"{type(error).__name__}: {error}"}
        torch.cuda.empty_cache()
    replicas.barrier(device)
    if reference_package() is not None:
        from helios_b200 import load

        stage("config 5")
        point = load.measure(CONFIG5_RATE, CONFIG5_REQUESTS_PER_GPU * size, device=device)
        stage("config 5 done")
        if rank == 0:
            point["workload"] = (f"BASELINE config 5 at {CONFIG5_RATE:g} req/s per GPU, "
                                 f"{CONFIG5_REQUESTS_PER_GPU} requests per GPU (the full sweep: "
                                 "python -m helios_b200.load)")
            out["config5"] = point
        torch.cuda.empty_cache()
        if rank == 0 and size == 1:
            stage("reference GPU dense path")
            out["reference_gpu_dense"] = reference_gpu_dense(device, steps=min(args.steps, 8))
    elif rank == 0:
        out["config5"] = out["reference_gpu_dense"] = {"unavailable": "the reference package is not importable "
                                                                      "(baseline/_ref or HELIOS_REFERENCE_SRC)"}
    replicas.barrier(device)
    return out


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=32)  # BASELINE config 3 times 32 consecutive ticks
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    parser.add_argument("--no-extras", action="store_true",
                        help="skip configs 4 and 5 and the reference's GPU path (headline tick only)")
    parser.add_argument("--decode-sms", type=int, default=None,
                        help="SMs the decode attention grid keeps beside prefill work (0: all; default: the library's)")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("at least 3 warm-up steps")
    if args.decode_sms is not None and args.impl == "b200":
        from helios_b200 import _native

        _native.check(_native.load().hb_attention_set_overlap(args.decode_sms), "hb_attention_set_overlap")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
