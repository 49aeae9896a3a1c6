"""Model configuration and sampling parameters (same fields as the reference).

``Qwen3Config`` mirrors src/helios/runtime/qwen3/config.py:8-20 and
``Sampling`` mirrors src/helios/runtime/types.py:4-7 (same names, defaults and
bounds), so code written against the reference constructs them unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

QWEN3_4B_MODEL_ID = "Qwen/Qwen3-4B"


@dataclass(frozen=True)
class Qwen3Config:
    vocab_size: int = 151_936
    context_length: int = 40_960
    hidden_size: int = 2_560
    n_heads: int = 32
    n_layers: int = 36
    hidden_dim: int = 9_728
    head_dim: int = 128
    n_kv_heads: int = 8
    rope_base: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    dtype: torch.dtype = torch.bfloat16


def qwen3_4b_config(dtype: torch.dtype = torch.bfloat16) -> Qwen3Config:
    return Qwen3Config(dtype=dtype)


@dataclass(frozen=True)
class Sampling:
    max_new_tokens: int = 256
    temperature: float = 0.2
    top_p: float = 0.95

    def __post_init__(self) -> None:
        if not 1 <= self.max_new_tokens <= 2_048:
            raise ValueError("max_new_tokens must be between 1 and 2048")
        if not 0 <= self.temperature <= 2:
            raise ValueError("temperature must be between 0 and 2")
        if not 0 < self.top_p <= 1:
            raise ValueError("top_p must be in (0, 1]")
