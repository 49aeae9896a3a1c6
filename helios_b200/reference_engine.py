"""The reference's serving engine over the B200 path.

The reference (sidmanale643/helios) builds its decoder and KV page pool inside
``Generator`` from two names imported into ``helios.runtime.generate``
(generate.py:64 ``Decoder(model)``, :84-86 ``KVPagePool(...)``), and its prefix cache
tells paged block snapshots from dense ones by class (prefix_cache.py:333). Pointing
those names at this package's ``Decoder``, ``KVPagePool`` and ``PagedKVBlockSnapshot``
is the whole swap: the reference's ``Engine`` (scheduler tick ``_continuous_tick``,
admission, ``_run_mixed_batch`` row selection, ``_execute_batch`` sampling and
speculative verification, engine.py:197-530), ``Generator``, ``PrefixCache`` and
``Scheduler`` then run unchanged, and every model forward of every tick goes through
the B200 kernels. A maintainer makes the same change as import lines in those two
modules; ``b200_path`` makes it at run time, for as long as the engine lives.

``build_engine`` constructs the reference ``Engine`` around a B200 ``Qwen3Model``
without the reference's HuggingFace loader or memory profiling: the caller states the
KV budget in pages. The reference package is found on ``sys.path``, else under
``$HELIOS_REFERENCE_SRC``, else in the repository's ``baseline/_ref`` install.
"""

from __future__ import annotations

import contextlib
import importlib
import os
import sys
from pathlib import Path

import torch

from helios_b200.decode import Decoder
from helios_b200.paged_cache import KVPagePool, PagedKVBlockSnapshot

_REPO = Path(__file__).resolve().parent.parent


class ReferenceUnavailable(ImportError):
    pass


def import_reference():
    """The reference's ``helios`` package (imported unchanged)."""
    try:
        return importlib.import_module("helios.runtime.engine")
    except ImportError:
        pass
    for candidate in (os.environ.get("HELIOS_REFERENCE_SRC"), str(_REPO / "baseline" / "_ref")):
        if candidate and (Path(candidate) / "helios" / "runtime" / "engine.py").is_file():
            if candidate not in sys.path:
                sys.path.append(candidate)
            try:
                return importlib.import_module("helios.runtime.engine")
            except ImportError as error:  # a dependency of the reference is missing
                raise ReferenceUnavailable(f"the reference at {candidate} does not import: {error}") from error
    raise ReferenceUnavailable("the reference package (helios) is not importable: set HELIOS_REFERENCE_SRC "
                               "or install it into baseline/_ref")


@contextlib.contextmanager
def b200_path():
    """Within the block, reference ``Generator``s build this package's ``Decoder`` and
    ``KVPagePool``, and the reference prefix cache accepts this package's paged snapshots
    (beside its own, so the reference's own paged path keeps working in the same process)."""
    import_reference()
    generate = importlib.import_module("helios.runtime.generate")
    prefix_cache = importlib.import_module("helios.runtime.prefix_cache")
    saved = (generate.Decoder, generate.KVPagePool, prefix_cache.PagedKVBlockSnapshot)
    reference_snapshot = saved[2] if isinstance(saved[2], type) else saved[2][0]
    generate.Decoder = Decoder
    generate.KVPagePool = KVPagePool
    # Only used in isinstance() there (prefix_cache.py:333), which accepts a tuple of classes.
    prefix_cache.PagedKVBlockSnapshot = (reference_snapshot, PagedKVBlockSnapshot)
    try:
        yield
    finally:
        generate.Decoder, generate.KVPagePool, prefix_cache.PagedKVBlockSnapshot = saved


class _Loader:
    """Stands in for the reference's ``Qwen3Loader`` (``load(config) -> LoadedQwen3``)."""

    def __init__(self, loaded) -> None:
        self.loaded = loaded

    def load(self, config):
        return self.loaded


def build_engine(model, *, kv_pages: int, max_batch_size: int = 128, prefill_chunk_size: int = 2048,
                 max_queue_size: int = 4096, speculative_tokens: int = 0, batch_wait_ms: float = 0.0,
                 scheduler_thread: bool = True, prefix_cache_ttl_seconds: float = 300.0):
    """A reference ``Engine`` whose decoder and page pool are this package's.

    ``model`` is a ``helios_b200.model.Qwen3Model`` on a CUDA device; ``kv_pages`` pages of
    256 tokens make up its KV budget (the reference derives it from a memory profile,
    check.py). With ``scheduler_thread=False`` the scheduler's worker thread is not started
    and the caller runs ticks with ``engine._continuous_tick(engine._scheduler)``, as the
    reference's own tests do (tests/test_continuous_batching.py:89-91). Call it inside
    ``b200_path()`` and keep the block open while the engine is used."""
    engine_module = import_reference()
    from helios.config import HeliosConfig
    from helios.runtime.check import CacheCapacity, MemoryReport
    from helios.runtime.qwen3.loader import LoadedQwen3

    config = model.config
    element = torch.empty((), dtype=config.dtype).element_size()
    bytes_per_token = config.n_layers * 2 * config.n_kv_heads * config.head_dim * element
    budget_tokens = kv_pages * 256
    budget_bytes = budget_tokens * bytes_per_token
    capacity = CacheCapacity(free_bytes=budget_bytes, device_occupied_bytes=0, activation_headroom_bytes=0,
                             bytes_per_token=bytes_per_token, max_tokens=min(budget_tokens, config.context_length),
                             kv_budget_bytes=budget_bytes, model_occupied_bytes=0)
    device = next(model.parameters()).device
    report = MemoryReport(gpu=torch.cuda.get_device_name(device) if device.type == "cuda" else device.type,
                          total_bytes=budget_bytes,
                          max_gpu_utilization=1.0, max_gpu_bytes=budget_bytes, free_before_load_bytes=budget_bytes,
                          weight_bytes=0, required_bytes=0, fits=True, cache=capacity)
    loader = _Loader(LoadedQwen3(model, capacity, report, "helios_b200"))
    helios_config = HeliosConfig(model_id="helios_b200", hf_token=None, max_batch_size=max_batch_size,
                                 prefill_chunk_size=prefill_chunk_size, max_queue_size=max_queue_size,
                                 speculative_tokens=speculative_tokens, batch_wait_ms=batch_wait_ms,
                                 prefix_cache_ttl_seconds=prefix_cache_ttl_seconds)
    if scheduler_thread:
        engine = engine_module.Engine(helios_config, loader=loader)
    else:
        from unittest.mock import patch

        with patch("helios.runtime.scheduler.Thread"):
            engine = engine_module.Engine(helios_config, loader=loader)
    if not isinstance(engine.generator.decoder, Decoder):
        raise RuntimeError("build_engine must run inside b200_path(): the engine built the reference decoder")
    return engine
