"""RMSNorm and RoPE oracle with the reference's rounding points.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

  * ``rms_norm`` -- ``RMSNorm.forward`` (src/helios/runtime/qwen3/layers.py:36-40):
    fp32 math, multiply by the fp32 scale, round to the input dtype.
  * ``rope_tables`` -- ``rope_parameters`` (layers.py:43-51).
  * ``apply_rope`` -- ``apply_rope`` with ``position_ids`` (layers.py:54-72):
    ``x*cos + rotate(x)*sin`` in fp32 from the already-rounded input, then round.
"""

from __future__ import annotations

import torch


def rms_norm(x: torch.Tensor, scale: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    normalized = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (normalized * scale.float()).to(x.dtype)


def rope_tables(head_dim: int, context_length: int, base: float) -> tuple[torch.Tensor, torch.Tensor]:
    exponents = torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim
    inverse = 1.0 / (base ** exponents)
    angles = torch.arange(context_length, dtype=torch.float32)[:, None] * inverse[None, :]
    angles = torch.cat((angles, angles), dim=1)
    return torch.cos(angles), torch.sin(angles)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """Rotate ``x[..., T, d]`` by the table rows at ``positions[T]``."""
    half = x.shape[-1] // 2
    c = cos[positions]
    s = sin[positions]
    while c.dim() < x.dim():
        c = c.unsqueeze(0)
        s = s.unsqueeze(0)
    rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return (x * c + rotated * s).to(x.dtype)
