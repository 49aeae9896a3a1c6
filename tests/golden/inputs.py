"""Seeded inputs shared by the fixture generator and the tests.

CPU ``torch.Generator`` streams are deterministic for a given PyTorch build, so
the fixtures store a SHA-256 of these tensors instead of the tensors; a test
that regenerates them checks the digest first.
"""

from __future__ import annotations

import hashlib

import torch


def attention_inputs(num_pages: int, tokens: int):
    """Seeded bf16 pool ``[P, 256, 1, 128]`` and packed q/k/v for the attention fixture."""
    g = torch.Generator().manual_seed(5)
    shape = (num_pages, 256, 1, 128)
    key_pool = (torch.randn(shape, generator=g) / 4).to(torch.bfloat16)
    value_pool = torch.randn(shape, generator=g).to(torch.bfloat16)
    q = torch.randn(1, 4, tokens, 128, generator=g).to(torch.bfloat16)
    k = (torch.randn(1, 1, tokens, 128, generator=g) / 4).to(torch.bfloat16)
    v = torch.randn(1, 1, tokens, 128, generator=g).to(torch.bfloat16)
    return key_pool, value_pool, q, k, v


def digest(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()
