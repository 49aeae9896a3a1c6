"""End-to-end parity at BASELINE config 3's model shape, against the reference.

``tests/golden/qwen3_4b_tick.npz`` was written by the reference's own packed CPU path
(src/helios/runtime/qwen3/decode.py:260-291, paged_cache.py:521-546) on the Qwen3-4B
architecture (36 layers, hidden 2560, 32/8 heads, d=128, inter 9728, vocab 151936, tied
embeddings) with its seed-0 bf16 weights: 8 decode rows whose prompts (contexts
U[1024, 4096]) it prefilled itself, then one packed tick of those rows plus a fresh
2048-token prefill chunk, then 63 greedy ticks. The B200 model gets the same weights
(redrawn in parallel from the generator states in ``qwen3_4b_init.npz`` and checked
against the digests of the reference's own initialisation), prefills the same prompts
through its own kernels and runs the same ticks: eager, with the greedy head fused into
the lm_head GEMM, and from CUDA graphs.

Tolerances are in bf16 units in the last place (ulp) of the row's largest logit: a
correct bf16 implementation differs from the reference by rounding only, and at the
logit magnitudes of this model (the winning logit is ~2000, ulp 8) an absolute bound
such as 2e-2 is below one ulp. Greedy ids must be identical at every step. With the
random-init weights and N(0, 1) tied embeddings, every row's greedy token is its own
last input (the embedding's self-product dominates the logits), so the logit values
carry most of the check; the runner-up margins are recorded to show no step is a near tie.
"""

from __future__ import annotations

import hashlib
import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

from helios_b200 import _native
from helios_b200.config import Qwen3Config
from helios_b200.decode import Decoder
from helios_b200.model import Qwen3Model
from helios_b200.paged_cache import KVPagePool, PagedKVCache
from oracle.model import OracleConfig, build_state_dict

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
LOGIT_ULPS = 2  # bound on |B200 - reference| in ulps of the row's largest logit


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bf16 values at magnitude |x| (8 significand bits)."""
    mag = np.maximum(np.abs(x), np.finfo(np.float32).tiny)
    return np.exp2(np.floor(np.log2(mag)) - 7)


def _split(flat, lengths):
    out, at = [], 0
    for n in lengths:
        out.append(flat[at:at + n])
        at += n
    return out


@pytest.fixture(scope="module")
def golden(golden_dir):
    return np.load(golden_dir / "qwen3_4b_tick.npz")


@pytest.fixture(scope="module")
def model(golden_dir):
    init = np.load(golden_dir / "qwen3_4b_init.npz")
    threads = max(4, os.cpu_count() or 4)
    states = [torch.from_numpy(s.copy()) for s in init["rng_states"]]
    sd = build_state_dict(OracleConfig(), 0, rng_checkpoints=states, threads=threads)
    names = [str(n) for n in init["names"]]

    def digest(name):
        return hashlib.sha256(sd[name].contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()

    with ThreadPoolExecutor(threads) as pool:
        got = list(pool.map(digest, names))
    bad = [n for n, g, w in zip(names, got, init["sha256"]) if g != str(w)]
    assert not bad, f"weights differ from the reference's seed-0 initialisation: {bad[:4]}"
    m = Qwen3Model.from_state_dict(Qwen3Config(), sd, DEV)
    del sd
    return m


def _prefilled(model, g):
    decoder = Decoder(model)
    steps = g["greedy"].shape[1]
    prompts = _split(g["prompts"].tolist(), g["prompt_lengths"].tolist())
    pages = sum(math.ceil((len(p) + 1 + steps) / 256) for p in prompts) + math.ceil((2048 + steps) / 256) + 4
    pool = decoder.page_pool = KVPagePool(model.config, pages, device=DEV)
    caches = []
    for prompt in prompts:
        cache = PagedKVCache(pool, len(prompt) + 1 + steps)
        decoder.packed_caches([cache], [prompt])
        caches.append(cache)
    caches.append(PagedKVCache(pool, 2048 + steps))
    return decoder, caches


def _check_logits(logits: torch.Tensor, g, label: str) -> float:
    got = logits.float().cpu().numpy()[:, g["columns"]]
    want = g["tick_logits"]
    # The row's largest logit is its winning one (the strided columns need not hold it).
    row_max = np.maximum(np.abs(g["greedy_max"][:, :1]), np.abs(want).max(-1, keepdims=True))
    err = np.abs(got - want) / bf16_ulp(row_max)
    print(f"[{label}] tick logits vs reference: max {err.max():.3f} ulp of the row max "
          f"(mean {err.mean():.4f}); abs max {np.abs(got - want).max():.4f}")
    assert err.max() <= LOGIT_ULPS, err.max(-1)
    return float(err.max())


def _run(model, g, *, greedy_head: bool, label: str):
    decoder, caches = _prefilled(model, g)
    pending = g["pending"].tolist()
    chunk = g["chunk"].tolist()
    steps = g["greedy"].shape[1]
    ids, best = [], []
    if greedy_head:
        ids.append(decoder.packed_caches_greedy(caches, [[t] for t in pending] + [chunk]).tolist())
    else:
        logits = decoder.packed_caches(caches, [[t] for t in pending] + [chunk])
        _check_logits(logits, g, label)
        ids.append(logits.argmax(-1).tolist())
        best.append(logits.float().max(-1).values.tolist())
    for step in range(1, steps):
        # The reference's own ids go in at every step, so one differing id could not
        # hide later ones; the ids we produce are compared below.
        feed = [[int(t)] for t in g["greedy"][:, step - 1]]
        if greedy_head:
            ids.append(decoder.packed_caches_greedy(caches, feed).tolist())
        else:
            out = decoder.packed_caches(caches, feed).float()
            ids.append(out.argmax(-1).tolist())
            best.append(out.max(-1).values.tolist())
    ids = np.array(ids).T
    mismatched = np.argwhere(ids != g["greedy"])
    assert mismatched.size == 0, f"[{label}] greedy ids differ at (row, step) {mismatched[:8].tolist()}"
    margin = (g["greedy_max"] - g["greedy_second"]).min()
    if best:
        best = np.array(best).T
        want = g["greedy_max"]
        err = np.abs(best - want) / bf16_ulp(want)
        print(f"[{label}] {steps} greedy steps identical; winning logit max {err.max():.3f} ulp; "
              f"smallest reference runner-up margin {margin:.1f}")
        assert err.max() <= LOGIT_ULPS
    else:
        print(f"[{label}] {steps} greedy steps identical (greedy head fused into the lm_head GEMM)")
    assert _native.device_status() == 0


def test_qwen3_4b_tick_and_64_greedy_steps_match_reference(model, golden):
    _run(model, golden, greedy_head=False, label="eager")


def test_qwen3_4b_fused_greedy_head_matches_reference(model, golden):
    _run(model, golden, greedy_head=True, label="greedy head")


def test_qwen3_4b_cuda_graph_ticks_match_reference(model, golden):
    model.enable_cuda_graphs()
    try:
        _run(model, golden, greedy_head=False, label="cuda graphs")
    finally:
        model._graphs = None
