"""The reference's Engine, unchanged, running its scheduler ticks over the B200 path.

``helios_b200.reference_engine.build_engine`` builds the reference's ``Engine`` whose
``Generator`` holds this package's ``Decoder`` and ``KVPagePool``; every tick the
reference's ``_continuous_tick`` (src/helios/runtime/engine.py:197-214) selects rows and
chunks, and every forward goes through the B200 kernels. Requests of several prompt
lengths (chunked prefill across ticks, mixed decode + prefill ticks), a request that
restores a prefix the prefix cache stored from an earlier one (page aliasing), a sampled
request and speculative drafts are driven to completion with synchronous ticks, as the
reference's own tests do (tests/test_continuous_batching.py:89-178). Greedy outputs must
equal (1) a standalone run of each request through the B200 ``Decoder.generate`` and
(2) the reference's own Engine running the same requests with the same weights on its
CPU path.

Skipped, with the reason printed, when the reference package is not on the box
(HELIOS_REFERENCE_SRC or baseline/_ref).
"""

from __future__ import annotations

import pytest
import torch

from helios_b200 import _native
from helios_b200.config import Qwen3Config
from helios_b200.decode import Decoder
from helios_b200.model import Qwen3Model
from helios_b200.paged_cache import KVPagePool
from oracle.model import OracleConfig, build_state_dict

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
SHAPE = dict(vocab_size=4096, context_length=4096, hidden_size=512, n_heads=8, n_layers=2, hidden_dim=1024,
             head_dim=128, n_kv_heads=2, rope_base=1e6, rms_norm_eps=1e-6, dtype=torch.bfloat16)
PAGES = 48
NEW_TOKENS = 12


@pytest.fixture(scope="module")
def reference():
    from helios_b200 import reference_engine

    try:
        reference_engine.import_reference()
    except reference_engine.ReferenceUnavailable as error:
        pytest.skip(f"reference engine not available on this box: {error}")
    return reference_engine


@pytest.fixture(scope="module")
def weights():
    return build_state_dict(OracleConfig(**SHAPE), 0)


def _prompts():
    g = torch.Generator().manual_seed(11)
    shared = torch.randint(1, SHAPE["vocab_size"], (512,), generator=g).tolist()
    return {
        "long": shared + torch.randint(1, SHAPE["vocab_size"], (90,), generator=g).tolist(),
        "short": torch.randint(1, SHAPE["vocab_size"], (40,), generator=g).tolist(),
        "mid": torch.randint(1, SHAPE["vocab_size"], (300,), generator=g).tolist(),
        "prefix_hit": shared + torch.randint(1, SHAPE["vocab_size"], (33,), generator=g).tolist(),
    }


def _drive(engine, sampling_cls, *, sampled: bool = True) -> dict:
    """First wave: long, short, mid (+ one sampled request); once ``long`` has finished and
    stored its blocks, ``prefix_hit`` restores them. Returns the results by name."""
    prompts = _prompts()
    greedy = sampling_cls(temperature=0, top_p=1, max_new_tokens=NEW_TOKENS)
    futures = {name: engine.enqueue(prompts[name], 0, greedy, request_id=name) for name in ("long", "short", "mid")}
    if sampled:
        futures["sampled"] = engine.enqueue(prompts["short"], 0,
                                            sampling_cls(temperature=0.7, top_p=0.9, max_new_tokens=NEW_TOKENS),
                                            request_id="sampled")
    for _ in range(400):
        if futures["long"].done():
            break
        engine._continuous_tick(engine._scheduler)
    futures["prefix_hit"] = engine.enqueue(prompts["prefix_hit"], 0, greedy, request_id="prefix_hit")
    for _ in range(400):
        if all(f.done() for f in futures.values()):
            break
        engine._continuous_tick(engine._scheduler)
    return {name: f.result(timeout=0) for name, f in futures.items()}


def _b200_engine(reference, weights, **kwargs):
    model = Qwen3Model.from_state_dict(Qwen3Config(**SHAPE), weights, DEV)
    return reference.build_engine(model, kv_pages=PAGES, max_batch_size=8, prefill_chunk_size=256,
                                  scheduler_thread=False, **kwargs)


def _standalone(weights, prompt):
    from helios_b200.config import Sampling

    model = Qwen3Model.from_state_dict(Qwen3Config(**SHAPE), weights, DEV)
    decoder = Decoder(model)
    decoder.page_pool = KVPagePool(model.config, PAGES, device=DEV)
    result = decoder.generate(prompt, 0, Sampling(temperature=0, top_p=1, max_new_tokens=NEW_TOKENS),
                              max_total_tokens=SHAPE["context_length"])
    decoder.release_cache(result.cache)
    return result.output_ids, result.finish_reason


def _reference_on_cpu(reference, weights):
    """The reference's own Engine, Decoder and paged CPU path, same weights and requests."""
    from unittest.mock import patch

    from helios.config import HeliosConfig
    from helios.runtime.check import CacheCapacity, MemoryReport
    from helios.runtime.engine import Engine
    from helios.runtime.qwen3.config import Qwen3Config as RefConfig
    from helios.runtime.qwen3.loader import LoadedQwen3
    from helios.runtime.qwen3.model import Qwen3Model as RefModel
    from helios.runtime.types import Sampling as RefSampling

    cfg = RefConfig(**SHAPE)
    torch.manual_seed(0)
    model = RefModel(cfg).eval()  # the reference's seed-0 weights, the ones ``weights`` restates
    assert all(torch.equal(model.state_dict()[k], v) for k, v in weights.items())
    bytes_per_token = cfg.n_layers * 2 * cfg.n_kv_heads * cfg.head_dim * 2
    budget = PAGES * 256 * bytes_per_token
    capacity = CacheCapacity(free_bytes=budget, device_occupied_bytes=0, activation_headroom_bytes=0,
                             bytes_per_token=bytes_per_token, max_tokens=min(PAGES * 256, cfg.context_length),
                             kv_budget_bytes=budget, model_occupied_bytes=0)
    report = MemoryReport(gpu="cpu", total_bytes=budget, max_gpu_utilization=1.0, max_gpu_bytes=budget,
                          free_before_load_bytes=budget, weight_bytes=0, required_bytes=0, fits=True, cache=capacity)

    class Loader:
        def load(self, config):
            return LoadedQwen3(model, capacity, report, "test")

    with patch("helios.runtime.scheduler.Thread"):
        engine = Engine(HeliosConfig(model_id="test", hf_token=None, max_batch_size=8, prefill_chunk_size=256,
                                     batch_wait_ms=0, max_queue_size=64), loader=Loader())
    try:
        return _drive(engine, RefSampling, sampled=False)
    finally:
        engine.close()


def test_reference_engine_over_b200_matches_standalone_and_reference(reference, weights):
    from helios.runtime.types import Sampling as RefSampling

    with reference.b200_path():
        engine = _b200_engine(reference, weights)
        try:
            results = _drive(engine, RefSampling)
            assert engine.generator.prefix_cache.blocks(), "the finished requests stored no prefix blocks"
        finally:
            engine.close()
    assert results["prefix_hit"].prefix.restored_tokens == 512
    assert results["long"].prefix.restored_tokens == 0
    sampled = results["sampled"]
    assert sampled.finish_reason in ("length", "eos") and all(0 <= t < SHAPE["vocab_size"] for t in sampled.output_ids)
    prompts = _prompts()
    for name in ("long", "short", "mid", "prefix_hit"):
        want = _standalone(weights, prompts[name])
        assert (results[name].output_ids, results[name].finish_reason) == want, name
    cpu = _reference_on_cpu(reference, weights)
    for name in ("long", "short", "mid", "prefix_hit"):
        assert results[name].output_ids == cpu[name].output_ids, name
        assert results[name].finish_reason == cpu[name].finish_reason, name
    assert cpu["prefix_hit"].prefix.restored_tokens == 512
    print("engine over B200 == standalone B200 == reference engine on CPU:",
          {name: results[name].output_ids[:4] for name in ("long", "short", "mid", "prefix_hit")})
    assert _native.device_status() == 0


def test_reference_engine_speculative_drafts_over_b200_match_plain_greedy(reference, weights):
    from helios.runtime.types import Sampling as RefSampling

    with reference.b200_path():
        plain = _b200_engine(reference, weights)
        try:
            want = _drive(plain, RefSampling, sampled=False)
        finally:
            plain.close()
        drafted = _b200_engine(reference, weights, speculative_tokens=4)
        try:
            got = _drive(drafted, RefSampling, sampled=False)
        finally:
            drafted.close()
    for name in want:
        assert got[name].output_ids == want[name].output_ids, name
    assert _native.device_status() == 0
