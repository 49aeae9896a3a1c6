"""Generate golden vectors from the reference implementation (sidmanale643/helios).

Run in a container that holds the reference sources:

    HELIOS_REFERENCE_SRC=<reference>/src python tests/golden/make_golden.py

It imports the reference *unchanged* and records, as small fixtures in this
directory, what its own code computes:

  metadata.json   -- ``PagedBatchCache.prepare`` / ``PackedBatchCache.prepare_packed``
                     outputs for the reference tests' known-answer cases
                     (tests/test_paged_attention.py:59-118, :253-263), BASELINE
                     config 1's tick, a config-3-shaped tick, drafted rows and a
                     restored prefix, with the page tables the reference's pool
                     handed out (LIFO).
  config1.npz     -- BASELINE config 1: tiny fp32 Qwen3 (seed 0) tick logits on the
                     reference's dense-KV path and on its packed CPU path, plus 16
                     greedy steps.
  bf16_tick.npz   -- a bf16 mixed tick at the Qwen3-4B head shape (d=128, 4 query
                     heads per KV head) on the reference's packed CPU path, plus 64
                     greedy decode steps.
  qwen3_4b_init.npz -- (``make_golden.py qwen3_4b_init``) digests of the reference's
                     seed-0 Qwen3-4B weights and the generator states that let a test
                     redraw them in parallel.
  qwen3_4b_tick.npz -- (``make_golden.py qwen3_4b_tick``) BASELINE config 3's model
                     (Qwen3-4B shape, seed-0 bf16) and tick shape on the reference's
                     packed CPU path: 8 prefilled decode rows plus a 2048-token chunk,
                     then 64 greedy steps.
  attention.npz   -- ``PackedBatchCache.attend`` (CPU branch) output for seeded bf16
                     inputs over decode, drafted and chunked-prefill rows.
  sampler.npz     -- kept token sets of ``Decoder._sample`` (captured from the
                     probabilities handed to ``torch.multinomial``) and greedy ids.

The GPU tests never read the reference; they read these files.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path
from unittest.mock import patch

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
src = os.environ.get("HELIOS_REFERENCE_SRC")
if not src:
    raise SystemExit("set HELIOS_REFERENCE_SRC to the reference's src/ directory")
sys.path.insert(0, src)

from helios.runtime.qwen3.cache import KVCache  # noqa: E402
from helios.runtime.qwen3.config import Qwen3Config  # noqa: E402
from helios.runtime.qwen3.decode import Decoder  # noqa: E402
from helios.runtime.qwen3.model import Qwen3Model  # noqa: E402
from helios.runtime.qwen3.paged_cache import (  # noqa: E402
    KVPagePool,
    PackedBatchCache,
    PagedBatchCache,
    PagedKVCache,
)
from helios.runtime.types import Sampling  # noqa: E402

from oracle.model import OracleConfig, build_state_dict, rng_checkpoints  # noqa: E402
from tests.golden.inputs import attention_inputs, digest  # noqa: E402

torch.set_num_threads(max(1, os.cpu_count() or 1))


def tiny_meta_config() -> Qwen3Config:
    """Metadata does not depend on head shapes; keep the pool small."""
    return Qwen3Config(vocab_size=64, context_length=40_960, hidden_size=16, n_heads=2, n_layers=1,
                       hidden_dim=32, head_dim=8, n_kv_heads=1, dtype=torch.float32)


def _lists(batch, names):
    return {name: getattr(batch, name).tolist() for name in names}


def metadata_cases() -> list[dict]:
    cases = []
    cfg = tiny_meta_config()
    cpu = torch.device("cpu")

    # tests/test_paged_attention.py:97-118 -- mixed lengths 3 and 7, then one decode token.
    pool = KVPagePool(cfg, 6, device=cpu)
    short, long = PagedKVCache(pool, 512), PagedKVCache(pool, 512)
    for cache, tokens in ((short, 3), (long, 7)):
        b = PagedBatchCache([cache]); b.prepare(tokens); b.advance(tokens)
    lengths = [short.length, long.length]
    b = PagedBatchCache([short, long]); b.prepare(1)
    cases.append({"name": "ref_mixed_lengths", "mode": "uniform", "tokens": 1, "lengths": lengths,
                  "capacities": [512, 512], "page_tables": [[p.index for p in c.pages] for c in (short, long)],
                  "expected": _lists(b, ["block_table", "seqused_k", "cu_seq_q", "cu_seq_k", "write_slots"])
                  | {"max_q": b.max_q, "max_k": b.max_k}})

    # tests/test_paged_attention.py:253-263 -- two empty caches, prefill of 2 tokens.
    pool = KVPagePool(cfg, 4, device=cpu)
    caches = [PagedKVCache(pool, 512), PagedKVCache(pool, 512)]
    b = PagedBatchCache(caches); b.prepare(2)
    cases.append({"name": "ref_prefill_two", "mode": "uniform", "tokens": 2, "lengths": [0, 0],
                  "capacities": [512, 512], "page_tables": [[p.index for p in c.pages] for c in caches],
                  "expected": _lists(b, ["block_table", "seqused_k", "cu_seq_q", "cu_seq_k", "write_slots"])
                  | {"max_q": b.max_q, "max_k": b.max_k}})

    # tests/test_paged_attention.py:59-74 -- 256 tokens fill one page, the 257th takes the next.
    pool = KVPagePool(cfg, 6, device=cpu)
    cache = PagedKVCache(pool, 512)
    b = PagedBatchCache([cache]); b.prepare(256)
    first = {"block_table": b.block_table.tolist(), "write_slots": b.write_slots.tolist()}
    b.advance(256)
    b = PagedBatchCache([cache]); b.prepare(1)
    cases.append({"name": "page_boundary", "mode": "uniform", "tokens": 1, "lengths": [256],
                  "capacities": [512], "page_tables": [[p.index for p in cache.pages]],
                  "first_prepare": first,
                  "expected": _lists(b, ["block_table", "seqused_k", "cu_seq_q", "cu_seq_k", "write_slots"])
                  | {"max_q": b.max_q, "max_k": b.max_k}})

    def packed_case(name, lengths, counts, capacities, logit_counts=None, pool_pages=64, restore=None):
        pool = KVPagePool(cfg, pool_pages, device=cpu)
        caches = []
        acquired_before = []
        snapshot = None
        if restore is not None:
            donor = PagedKVCache(pool, restore + 1)
            b = PagedBatchCache([donor]); b.prepare(restore); b.advance(restore)
            snapshot = donor.snapshot_block(0, restore)
            donor.close()
        for length, cap in zip(lengths, capacities):
            c = PagedKVCache(pool, cap)
            if snapshot is not None and length == restore:
                c.restore_blocks([snapshot])
            elif length:
                b = PagedBatchCache([c]); b.prepare(length); b.advance(length)
            caches.append(c)
            acquired_before.append([p.index for p in c.pages])
        packed = PackedBatchCache(caches)
        packed.prepare_packed(counts, logit_counts)
        return {"name": name, "mode": "packed", "lengths": lengths, "counts": counts,
                "logit_counts": logit_counts, "capacities": capacities,
                "pages_before": acquired_before,
                "page_tables": [[p.index for p in c.pages] for c in caches],
                "expected": _lists(packed, ["block_table", "cu_seq_q", "cu_seq_k", "seqused_k",
                                            "positions", "logit_indices", "write_slots"])
                | {"max_q": packed.max_q, "max_k": packed.max_k}}

    # decode rows at 37/120/255/300 plus a 200-token prefill at offset 0.
    cases.append(packed_case("config1_tick", [37, 120, 255, 300, 0], [1, 1, 1, 1, 200],
                             [37 + 17, 120 + 17, 255 + 17, 300 + 17, 200 + 16], pool_pages=16))
    # A config-3-shaped tick: 32 decode rows with contexts in [1024, 4096] + a 2048-token prefill.
    g = torch.Generator().manual_seed(3)
    ctx = torch.randint(1024, 4097, (32,), generator=g).tolist()
    lengths = [c - 1 for c in ctx] + [0]
    counts = [1] * 32 + [2048]
    caps = [c + 63 for c in ctx] + [2048 + 64]
    cases.append(packed_case("config3_tick", lengths, counts, caps, pool_pages=700))
    # Drafted decode rows (speculative verification): several logit rows per sequence.
    cases.append(packed_case("drafted_rows", [10, 300, 0], [3, 5, 40], [64, 400, 64],
                             logit_counts=[3, 5, 1], pool_pages=16))
    # Chunked prefill continuing at a page boundary and mid-page.
    cases.append(packed_case("chunked_prefill", [256, 100, 511], [300, 156, 2], [1024, 300, 600],
                             pool_pages=32))
    # A row restored from a 512-token prefix snapshot by page aliasing, then extended.
    cases.append(packed_case("restored_prefix", [512, 7], [40, 1], [700, 64], pool_pages=16, restore=512))
    return cases


def rand_ids(generator, n, vocab):
    return torch.randint(0, vocab, (n,), generator=generator).tolist()


def config1() -> dict:
    cfg = Qwen3Config(vocab_size=4096, context_length=4096, hidden_size=256, n_heads=4, n_layers=2,
                      hidden_dim=768, head_dim=64, n_kv_heads=2, rope_base=1e6, rms_norm_eps=1e-6,
                      dtype=torch.float32)
    torch.manual_seed(0)
    model = Qwen3Model(cfg).eval()
    ocfg = OracleConfig(**{k: getattr(cfg, k) for k in OracleConfig.__dataclass_fields__})
    sd = build_state_dict(ocfg, 0)
    ref_sd = model.state_dict()
    weights_match = all(torch.equal(ref_sd[k], sd[k]) for k in sd)
    g = torch.Generator().manual_seed(0)
    contexts = [37, 120, 255, 300]
    prompts = [rand_ids(g, c, cfg.vocab_size) for c in contexts]
    pending = rand_ids(g, 4, cfg.vocab_size)
    chunk = rand_ids(g, 200, cfg.vocab_size)
    steps = 16
    with torch.inference_mode():
        dense = []
        for prompt in prompts:
            cache = KVCache(cfg, len(prompt) + steps + 1, device=torch.device("cpu"))
            model(torch.tensor([prompt]), cache=cache)
            dense.append(cache)
        prefill_cache = KVCache(cfg, 200 + steps, device=torch.device("cpu"))
        logits = [model(torch.tensor([[tok]]), cache=c)[0, -1] for tok, c in zip(pending, dense)]
        logits.append(model(torch.tensor([chunk]), cache=prefill_cache)[0, -1])
        logits = torch.stack(logits)
        caches = dense + [prefill_cache]
        tokens = [logits.argmax(-1).tolist()]
        for _ in range(steps - 1):
            nxt = [model(torch.tensor([[t]]), cache=c)[0, -1].argmax().item() for t, c in zip(tokens[-1], caches)]
            tokens.append(nxt)
        # The same tick on the reference's packed paged CPU path.
        pool = KVPagePool(cfg, 16, device=torch.device("cpu"))
        paged = []
        for prompt in prompts:
            pc = PagedKVCache(pool, len(prompt) + steps + 1)
            b = PagedBatchCache([pc]); b.prepare(len(prompt)); model(torch.tensor([prompt]), cache=b)
            paged.append(pc)
        paged.append(PagedKVCache(pool, 200 + steps))
        decoder = Decoder(model)
        decoder.page_pool = pool
        packed_logits = decoder.packed_caches(paged, [[t] for t in pending] + [chunk])
    return {
        "prompt_lengths": np.array(contexts), "prompts": np.concatenate([np.array(p) for p in prompts]),
        "pending": np.array(pending), "chunk": np.array(chunk),
        "dense_logits": logits.numpy(),
        "packed_vs_dense_max_abs": np.array(float((packed_logits - logits).abs().max())),
        "greedy": np.array(tokens).T, "weights_match": np.array(weights_match),
        "embedding_sum": np.array(float(ref_sd["token_embedding.weight"].double().sum())),
    }


BF16_SHAPE = dict(vocab_size=4096, context_length=4096, hidden_size=512, n_heads=8, n_layers=2,
                  hidden_dim=1024, head_dim=128, n_kv_heads=2, rope_base=1e6, rms_norm_eps=1e-6,
                  dtype=torch.bfloat16)


def bf16_tick() -> dict:
    """Mixed tick: decode rows at 100/300/600, a drafted row, a fresh prefill and a continued chunk."""
    cfg = Qwen3Config(**BF16_SHAPE)
    torch.manual_seed(0)
    model = Qwen3Model(cfg).eval()
    g = torch.Generator().manual_seed(1)
    contexts = [100, 300, 600, 256]
    prompts = [rand_ids(g, c, cfg.vocab_size) for c in contexts]
    chunks = [rand_ids(g, 1, cfg.vocab_size), rand_ids(g, 1, cfg.vocab_size), rand_ids(g, 3, cfg.vocab_size),
              rand_ids(g, 150, cfg.vocab_size), rand_ids(g, 300, cfg.vocab_size)]
    logit_counts = [1, 1, 3, 1, 1]
    steps = 64
    pool = KVPagePool(cfg, 24, device=torch.device("cpu"))
    decoder = Decoder(model)
    decoder.page_pool = pool
    with torch.inference_mode():
        caches = []
        for prompt in prompts:
            pc = PagedKVCache(pool, len(prompt) + 320 + steps)
            b = PagedBatchCache([pc]); b.prepare(len(prompt)); model(torch.tensor([prompt]), cache=b)
            caches.append(pc)
        caches.append(PagedKVCache(pool, 300 + steps))
        logits = decoder.packed_caches(caches, chunks, logit_counts=logit_counts)
        last_rows = np.cumsum(logit_counts) - 1
        heads = logits[torch.as_tensor(last_rows)].float()
        tokens = [heads.argmax(-1).tolist()]
        maxima = [heads.max(-1).values.tolist()]
        for _ in range(steps - 1):
            out = decoder.packed_caches(caches, [[t] for t in tokens[-1]]).float()
            tokens.append(out.argmax(-1).tolist())
            maxima.append(out.max(-1).values.tolist())
    return {
        "prompt_lengths": np.array(contexts), "prompts": np.concatenate([np.array(p) for p in prompts]),
        "chunk_lengths": np.array([len(c) for c in chunks]),
        "chunks": np.concatenate([np.array(c) for c in chunks]),
        "logit_counts": np.array(logit_counts),
        "logits": logits.float().numpy(), "greedy": np.array(tokens).T,
        "greedy_max": np.array(maxima, dtype=np.float32).T,
        "page_tables": np.array([p.index for c in caches for p in c.pages]),
        "page_counts": np.array([len(c.pages) for c in caches]),
    }


def qwen3_4b_tick(steps: int = 64, rows: int = 8) -> dict:
    """BASELINE config 3's model and tick shape on the reference's packed CPU path.

    Qwen3-4B architecture (36 layers, hidden 2560, 32/8 heads, d=128, inter 9728, vocab
    151936, tied), random-init bf16 from seed 0. ``rows`` decode rows whose prompts
    (contexts U[1024, 4096], seed 3) are prefilled through the reference's own paged
    path, then one packed tick of those rows' pending tokens plus a fresh 2048-token
    prefill chunk at offset 0, then ``steps - 1`` greedy decode ticks of all rows.
    Recorded: the tick's logits at every 37th vocabulary column, and per step and row
    the greedy id, the winning logit and the runner-up logit (so a test can tell a
    decided step from a near tie)."""
    import time

    cfg = Qwen3Config()
    started = time.time()
    torch.manual_seed(0)
    model = Qwen3Model(cfg).eval()
    print(f"init {time.time() - started:.1f} s", flush=True)
    g = torch.Generator().manual_seed(3)
    contexts = torch.randint(1024, 4097, (rows,), generator=g).tolist()
    prompts = [rand_ids(g, c, cfg.vocab_size) for c in contexts]
    pending = rand_ids(g, rows, cfg.vocab_size)
    chunk = rand_ids(g, 2048, cfg.vocab_size)
    pages = sum(-(-(c + steps + 1) // 256) for c in contexts) + -(-(2048 + steps) // 256) + 4
    pool = KVPagePool(cfg, pages, device=torch.device("cpu"))
    decoder = Decoder(model)
    decoder.page_pool = pool
    columns = np.arange(0, cfg.vocab_size, 37)
    with torch.inference_mode():
        caches = []
        for prompt in prompts:
            pc = PagedKVCache(pool, len(prompt) + 1 + steps)
            decoder.packed_caches([pc], [prompt])
            caches.append(pc)
            print(f"prefilled {len(prompt)} at {time.time() - started:.1f} s", flush=True)
        caches.append(PagedKVCache(pool, 2048 + steps))
        logits = decoder.packed_caches(caches, [[t] for t in pending] + [chunk]).float()
        print(f"tick at {time.time() - started:.1f} s", flush=True)
        tick_logits = logits[:, torch.as_tensor(columns)].numpy()
        ids, best, second = [], [], []

        def record(out):
            top = out.topk(2, dim=-1)
            ids.append(out.argmax(-1).tolist())
            best.append(top.values[:, 0].tolist())
            second.append(top.values[:, 1].tolist())

        record(logits)
        for step in range(steps - 1):
            record(decoder.packed_caches(caches, [[t] for t in ids[-1]]).float())
            if step % 8 == 7:
                print(f"step {step + 2} at {time.time() - started:.1f} s", flush=True)
    return {
        "prompt_lengths": np.array(contexts), "prompts": np.concatenate([np.array(p) for p in prompts]).astype(np.int32),
        "pending": np.array(pending, dtype=np.int32), "chunk": np.array(chunk, dtype=np.int32),
        "columns": columns.astype(np.int32), "tick_logits": tick_logits.astype(np.float32),
        "greedy": np.array(ids, dtype=np.int32).T, "greedy_max": np.array(best, dtype=np.float32).T,
        "greedy_second": np.array(second, dtype=np.float32).T,
        "page_counts": np.array([len(c.pages) for c in caches]),
    }


def qwen3_4b_init() -> dict:
    """The reference's seed-0 Qwen3-4B weights, as SHA-256 digests per tensor, and the CPU
    generator's state before the embedding and before each block, so a test can redraw the
    weights on many threads (``oracle.model.build_state_dict(rng_checkpoints=...)``) in
    seconds and prove them bit-identical to the reference's serial initialisation."""
    import hashlib

    cfg = Qwen3Config()
    torch.manual_seed(0)
    sd = Qwen3Model(cfg).state_dict()
    names = [k for k in sd if k not in ("cos", "sin")]
    digests = [hashlib.sha256(sd[k].contiguous().view(torch.uint8).numpy().tobytes()).hexdigest() for k in names]
    ocfg = OracleConfig(**{k: getattr(cfg, k) for k in OracleConfig.__dataclass_fields__})
    states = torch.stack(rng_checkpoints(ocfg, 0)).numpy()
    return {"names": np.array(names), "sha256": np.array(digests), "rng_states": states}


def attention_case() -> dict:
    """``PackedBatchCache.attend`` CPU branch on seeded bf16 inputs (group 4, d=128)."""
    cfg = Qwen3Config(vocab_size=64, context_length=4096, hidden_size=64, n_heads=4, n_layers=1,
                      hidden_dim=64, head_dim=128, n_kv_heads=1, dtype=torch.bfloat16)
    pool = KVPagePool(cfg, 12, device=torch.device("cpu"))
    lengths, counts = [300, 513, 0, 256], [1, 4, 40, 30]
    key_pool, value_pool, q, k, v = attention_inputs(12, sum(counts))
    pool.keys[0].copy_(key_pool)
    pool.values[0].copy_(value_pool)
    caches = []
    for length, count in zip(lengths, counts):
        c = PagedKVCache(pool, length + count + 8)
        if length:
            c.pages.extend(pool.acquire(-(-length // 256)))
            c.length = length
        caches.append(c)
    packed = PackedBatchCache(caches)
    packed.prepare_packed(counts)
    with torch.inference_mode():
        out = packed.attend(0, q, k, v)
    return {
        "lengths": np.array(lengths), "counts": np.array(counts),
        "block_table": packed.block_table.numpy(), "cu_seq_q": packed.cu_seq_q.numpy(),
        "seqused_k": packed.seqused_k.numpy(), "write_slots": packed.write_slots.numpy(),
        "num_pages": np.array(12), "input_sha256": np.array(digest(key_pool, value_pool, q, k, v)),
        "out": out.contiguous().view(torch.int16).numpy(),
    }


def sampler_cases() -> dict:
    g = torch.Generator().manual_seed(7)
    vocab = 4096
    rows = []
    for scale in (0.5, 2.0, 6.0):
        rows.append((torch.randn(vocab, generator=g) * scale).to(torch.bfloat16).float())
    tie = torch.zeros(vocab)
    tie[[17, 900, 3000]] = 5.0
    rows.append(tie)
    logits = torch.stack(rows)
    out = {"logits": logits.to(torch.bfloat16).view(torch.int16).numpy(), "temperature": [], "top_p": [], "kept": []}
    out["greedy"] = Decoder._sample(logits, Sampling(temperature=0, top_p=1, max_new_tokens=1)).reshape(-1).numpy()
    for temperature in (0.2, 0.7, 1.0, 1.5):
        for top_p in (0.5, 0.9, 0.95, 1.0):
            captured = {}
            real_sort = torch.sort

            def fake_multinomial(probs, num_samples):
                captured["probs"] = probs.clone()
                return torch.zeros(probs.shape[0], 1, dtype=torch.long)

            def spy_sort(x, descending=False):
                values, indices = real_sort(x, descending=descending)
                captured["order"] = indices.clone()
                return values, indices

            with patch("torch.multinomial", fake_multinomial), patch("torch.sort", spy_sort):
                Decoder._sample(logits, Sampling(temperature=temperature, top_p=top_p, max_new_tokens=1))
            probs = captured["probs"]
            if "order" in captured:
                kept = torch.zeros_like(probs, dtype=torch.bool)
                kept.scatter_(-1, captured["order"], probs > 0)
            else:
                kept = probs > 0
            out["temperature"].append(temperature)
            out["top_p"].append(top_p)
            out["kept"].append(np.packbits(kept.numpy(), axis=-1))
    return {k: np.array(v) for k, v in out.items()}


def main() -> None:
    if sys.argv[1:] == ["qwen3_4b_tick"]:
        # Minutes of CPU work (the reference's bf16 forward of ~22k prompt tokens at the
        # Qwen3-4B shape), so it is written on request only.
        np.savez_compressed(HERE / "qwen3_4b_tick.npz", **qwen3_4b_tick())
        return
    if sys.argv[1:] == ["qwen3_4b_init"]:
        np.savez_compressed(HERE / "qwen3_4b_init.npz", **qwen3_4b_init())
        return
    (HERE / "metadata.json").write_text(json.dumps(metadata_cases()))
    np.savez_compressed(HERE / "config1.npz", **config1())
    np.savez_compressed(HERE / "bf16_tick.npz", **bf16_tick())
    np.savez_compressed(HERE / "attention.npz", **attention_case())
    np.savez_compressed(HERE / "sampler.npz", **sampler_cases())
    for f in sorted(HERE.iterdir()):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
