"""helios_b200: a B200-native (sm_100a) packed mixed-batch forward for Helios.

The Python layer mirrors the reference's interface for this path
(``KVPagePool``, ``PagedKVCache``, ``PagedBatchCache``, ``PackedBatchCache``,
``Qwen3Model``, ``Decoder``); the compute runs in ``libhelios_b200.so``, hand-written
CUDA called through a C ABI (``include/helios_b200.h``). There is no CPU fallback:
ops raise when the library is missing or the tensors are not on a CUDA device.
"""

from helios_b200.config import Qwen3Config, Sampling, qwen3_4b_config
from helios_b200.paged_cache import (
    KVPage,
    KVPagePool,
    PackedBatchCache,
    PagedBatchCache,
    PagedKVBlockSnapshot,
    PagedKVCache,
)

__all__ = [
    "KVPage",
    "KVPagePool",
    "PackedBatchCache",
    "PagedBatchCache",
    "PagedKVBlockSnapshot",
    "PagedKVCache",
    "Qwen3Config",
    "Sampling",
    "qwen3_4b_config",
]
